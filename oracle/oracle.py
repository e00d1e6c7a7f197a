"""ctypes front end for the CPU oracle (oracle/forge_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs
import this module; the B200 product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None


def build() -> str:
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class OrcConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("context_length", C.c_int32),
                ("d_model", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32)]


class OrcRandom(C.Structure):
    _fields_ = [("seed_array", C.c_int32 * 56), ("inext", C.c_int32), ("inextp", C.c_int32)]


_F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_F64P = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_U32P = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.orc_random_init.argtypes = [C.POINTER(OrcRandom), C.c_int32]
        L.orc_random_next_double.argtypes = [C.POINTER(OrcRandom)]
        L.orc_random_next_double.restype = C.c_double
        L.orc_random_next_doubles.argtypes = [C.POINTER(OrcRandom), _F64P, C.c_int64]
        L.orc_param_count.argtypes = [C.POINTER(OrcConfig)]
        L.orc_param_count.restype = C.c_int32
        L.orc_param_numel.argtypes = [C.POINTER(OrcConfig), C.c_int32]
        L.orc_param_numel.restype = C.c_int64
        L.orc_total_params.argtypes = [C.POINTER(OrcConfig)]
        L.orc_total_params.restype = C.c_int64
        L.orc_param_name.argtypes = [C.POINTER(OrcConfig), C.c_int32, C.c_char_p, C.c_int32]
        L.orc_model_init.argtypes = [C.POINTER(OrcConfig), C.c_int32, C.POINTER(C.c_void_p)]
        L.orc_forward.argtypes = [C.POINTER(OrcConfig), C.POINTER(C.c_void_p), _I32P, C.c_int32, _F32P]
        L.orc_forward.restype = C.c_int32
        L.orc_forward_last.argtypes = L.orc_forward.argtypes
        L.orc_forward_last.restype = C.c_int32
        L.orc_greedy.argtypes = [_F32P, C.c_int32]
        L.orc_greedy.restype = C.c_int32
        L.orc_sample.argtypes = [_F32P, C.c_int32, C.c_float, C.c_int32, C.c_double]
        L.orc_sample.restype = C.c_int32
        L.orc_apply_repetition_controls.argtypes = [_F32P, C.c_int32, _I32P, C.c_int32, C.c_float, C.c_int32]
        L.orc_apply_repetition_controls.restype = C.c_int32
        L.orc_sample_step.argtypes = [_F32P, C.c_int32, _I32P, C.c_int32, C.c_float, C.c_int32,
                                      C.c_float, C.c_int32, C.POINTER(OrcRandom)]
        L.orc_sample_step.restype = C.c_int32
        L.orc_generate.argtypes = [C.POINTER(OrcConfig), C.POINTER(C.c_void_p), _I32P, C.c_int32, C.c_int32,
                                   C.c_float, C.c_int32, C.POINTER(OrcRandom), C.c_int32, C.c_float,
                                   C.c_int32, _I32P, C.c_void_p]
        L.orc_generate.restype = C.c_int32
        L.orc_generate_uniforms.argtypes = [C.POINTER(OrcConfig), C.POINTER(C.c_void_p), _I32P, C.c_int32,
                                            C.c_int32, C.c_float, C.c_int32, _F64P, C.c_int32, C.c_float,
                                            C.c_int32, _I32P, C.c_void_p]
        L.orc_generate_uniforms.restype = C.c_int32
        L.orc_gelu_array.argtypes = [_F32P, _F32P, C.c_int64]
        L.orc_layer_norm_rows.argtypes = [_F32P, _F32P, _F32P, _F32P, C.c_int32, C.c_int32]
        L.orc_softmax_rows.argtypes = [_F32P, C.c_int32, C.c_int32]
        L.orc_set_threads.argtypes = [C.c_int32]
        L.orc_get_threads.restype = C.c_int32
        L.orc_expf_array.argtypes = [_F32P, _F32P, C.c_int64]
        L.orc_expf_vs_double_scan.argtypes = [C.c_uint32, C.c_uint32, _U32P, C.c_int64]
        L.orc_expf_vs_double_scan.restype = C.c_int64
        L.orc_expf_hash.argtypes = [C.c_uint32, C.c_int32, np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")]
        _lib = L
    return _lib


# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Config:
    """ModelConfig (src/LLM.Core/Model/ModelConfig.cs:8-26)."""
    vocab_size: int
    context_length: int
    d_model: int
    n_layers: int
    n_heads: int

    def c(self) -> OrcConfig:
        return OrcConfig(self.vocab_size, self.context_length, self.d_model, self.n_layers, self.n_heads)


class DotNetRandom:
    """System.Random(seed) compat stream (published algorithm; parity unpinned)."""

    def __init__(self, seed: int):
        self._s = OrcRandom()
        lib().orc_random_init(C.byref(self._s), int(seed))

    def next_double(self) -> float:
        return lib().orc_random_next_double(C.byref(self._s))

    def next_doubles(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float64)
        lib().orc_random_next_doubles(C.byref(self._s), out, n)
        return out

    @property
    def state(self) -> OrcRandom:
        return self._s


def param_names(cfg: Config) -> list[str]:
    c = cfg.c()
    n = lib().orc_param_count(C.byref(c))
    buf = C.create_string_buffer(128)
    out = []
    for i in range(n):
        lib().orc_param_name(C.byref(c), i, buf, 128)
        out.append(buf.value.decode())
    return out


def param_shapes(cfg: Config) -> list[tuple[int, ...]]:
    D, F = cfg.d_model, 4 * cfg.d_model
    shapes = [(cfg.vocab_size, D), (cfg.context_length, D)]
    for _ in range(cfg.n_layers):
        shapes += [(D,), (D,), (D, 3 * D), (3 * D,), (D, D), (D,), (D,), (D,), (D, F), (F,), (F, D), (D,)]
    shapes += [(D,), (D,)]
    return shapes


def init_params(cfg: Config, seed: int) -> list[np.ndarray]:
    """GptModel(cfg, backend, new Random(seed)) weights, registration order."""
    params = [np.empty(s, np.float32) for s in param_shapes(cfg)]
    ptrs = (C.c_void_p * len(params))(*[p.ctypes.data for p in params])
    c = cfg.c()
    lib().orc_model_init(C.byref(c), int(seed), ptrs)
    return params


def round_bf16(cfg: Config, params) -> list[np.ndarray]:
    """The weights a FB2_WEIGHTS_BF16 model computes with: tok_emb and each
    layer's attn.qkv.w, attn.proj.w, mlp.fc.w, mlp.proj.w rounded to the
    nearest bf16 (ties to even); everything else unchanged.  (The reference
    keeps fp32; this is the oracle of the library's bf16 option.)"""
    out = [np.array(p, np.float32, copy=True) for p in params]
    idx = [0] + [2 + 12 * layer + j for layer in range(cfg.n_layers) for j in (2, 4, 8, 10)]
    for i in idx:
        u = out[i].view(np.uint32)
        finite = (u & np.uint32(0x7F800000)) != np.uint32(0x7F800000)
        r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
        u[finite] = r[finite]
    return out


def _ptrs(params):
    for p in params:
        assert p.dtype == np.float32 and p.flags.c_contiguous
    return (C.c_void_p * len(params))(*[p.ctypes.data for p in params])


def forward(cfg: Config, params, tokens) -> np.ndarray:
    toks = np.ascontiguousarray(tokens, np.int32)
    out = np.empty((len(toks), cfg.vocab_size), np.float32)
    c = cfg.c()
    rc = lib().orc_forward(C.byref(c), _ptrs(params), toks, len(toks), out)
    if rc != 0:
        raise ValueError("oracle forward rejected its arguments")
    return out


def forward_last(cfg: Config, params, tokens) -> np.ndarray:
    toks = np.ascontiguousarray(tokens, np.int32)
    out = np.empty(cfg.vocab_size, np.float32)
    c = cfg.c()
    rc = lib().orc_forward_last(C.byref(c), _ptrs(params), toks, len(toks), out)
    if rc != 0:
        raise ValueError("oracle forward rejected its arguments")
    return out


def greedy(logits) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    return lib().orc_greedy(x, len(x))


def sample(logits, temperature: float, top_k: int, u: float) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    if x.size == 0:
        raise ValueError("Need at least one logit.")
    r = lib().orc_sample(x, len(x), temperature, top_k, u)
    if r < 0:
        raise ValueError("invalid sampling options")
    return r


def apply_repetition_controls(logits, history, penalty: float, ngram: int) -> np.ndarray:
    x = np.array(logits, np.float32, copy=True)
    h = np.ascontiguousarray(history, np.int32)
    if h.size == 0:
        h = np.zeros(1, np.int32)
        n = 0
    else:
        n = len(h)
    rc = lib().orc_apply_repetition_controls(x, len(x), h, n, penalty, ngram)
    if rc != 0:
        raise ValueError("Repetition penalty must be finite and >= 1; n-gram size >= 0.")
    return x


def sample_step(logits, window, temperature, top_k, penalty, ngram, rng: DotNetRandom) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    w = np.ascontiguousarray(window, np.int32)
    r = lib().orc_sample_step(x, len(x), w, len(w), temperature, top_k, penalty, ngram, C.byref(rng.state))
    if r < 0:
        raise ValueError("invalid sampling options")
    return r


def generate(cfg: Config, params, prompt, max_new: int, temperature: float, top_k: int,
             rng: DotNetRandom | None = None, eos_id: int = -1, repetition_penalty: float = 1.0,
             no_repeat_ngram: int = 0, uniforms=None, return_logits: bool = False):
    """Sampler.Generate with the reference algorithm (full re-forward per token)."""
    p = np.ascontiguousarray(prompt, np.int32)
    out = np.empty(max(max_new, 1), np.int32)
    logits = np.empty((max(max_new, 1), cfg.vocab_size), np.float32) if return_logits else None
    lp = logits.ctypes.data if logits is not None else None
    c = cfg.c()
    if uniforms is not None:
        u = np.ascontiguousarray(uniforms, np.float64)
        n = lib().orc_generate_uniforms(C.byref(c), _ptrs(params), p, len(p), max_new, temperature, top_k,
                                        u, eos_id, repetition_penalty, no_repeat_ngram, out, lp)
    else:
        assert rng is not None
        n = lib().orc_generate(C.byref(c), _ptrs(params), p, len(p), max_new, temperature, top_k,
                               C.byref(rng.state), eos_id, repetition_penalty, no_repeat_ngram, out, lp)
    if n < 0:
        raise ValueError("oracle generate rejected its arguments")
    if return_logits:
        return out[:n].copy(), logits[:n].copy()
    return out[:n].copy()


def gelu(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_gelu_array(x, y, x.size)
    return y


def layer_norm(x, w, b) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_layer_norm_rows(x, np.ascontiguousarray(w, np.float32), np.ascontiguousarray(b, np.float32),
                              out, x.shape[0], x.shape[1])
    return out


def softmax_rows(x) -> np.ndarray:
    y = np.array(x, np.float32, copy=True)
    lib().orc_softmax_rows(y, y.shape[0], y.shape[1])
    return y


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


def expf(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_expf_array(x, y, x.size)
    return y


def expf_vs_double_scan(lo_bits: int, hi_bits: int, max_out: int = 1 << 16):
    out = np.zeros(max_out, np.uint32)
    n = lib().orc_expf_vs_double_scan(lo_bits, hi_bits, out, max_out)
    return n, out[:min(n, max_out)]


def expf_hash(lo_bits: int, nchunks: int) -> np.ndarray:
    out = np.zeros(nchunks, np.uint64)
    lib().orc_expf_hash(lo_bits, nchunks, out)
    return out
