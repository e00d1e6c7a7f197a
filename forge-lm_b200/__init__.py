"""forge-lm B200 backend: Python host mirror of ForgeLM's decode interface.

The reference (TitanUranus67/forge-lm, C#) runs its token loop as
`Sampler.Generate(model, prompt, maxNewTokens, temperature, topK, rng, eosId,
repetitionPenalty, noRepeatNgramSize)` (src/LLM.Core/Inference/Sampler.cs:78-109)
over `GptModel.ForwardLast` (src/LLM.Core/Model/GptModel.cs:202-209).  This
package exposes the same operations, with the same argument meanings and
validation, on top of libforge_b200.so (hand-written sm_100a kernels, C ABI in
include/forge_b200.h).  Everything computes on the GPU; nothing here falls
back to host arithmetic.

Exceptions: ArgumentException / ArgumentOutOfRangeException of the
reference surface as `ArgumentError` (a ValueError); device failures as
`NativeError`.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, Iterable, Sequence

import numpy as np

from . import _native as N
from ._native import ArgumentError, InvalidDataError, NativeError
from .dotnet_random import DotNetRandom

__all__ = ["ModelConfig", "B200Backend", "Sampler", "DotNetRandom", "ArgumentError", "NativeError",
           "InvalidDataError", "param_names", "param_shapes", "init_params", "device_count", "library_path",
           "read_forgemodel_header", "write_forgemodel", "BpeTokenizer"]


def library_path() -> str:
    return N.LIB_PATH


def device_count() -> int:
    n = C.c_int32(0)
    N.check(N.load().fb2_device_count(C.byref(n)))
    return n.value


@dataclass(frozen=True)
class ModelConfig:
    """ModelConfig (src/LLM.Core/Model/ModelConfig.cs:8-26)."""
    vocab_size: int
    context_length: int
    d_model: int
    n_layers: int
    n_heads: int

    def __post_init__(self):
        for name in ("vocab_size", "context_length", "d_model", "n_layers", "n_heads"):
            if getattr(self, name) <= 0:
                raise ArgumentError(N.FB2_INVALID_ARG, f"{name} must be positive.")
        if self.d_model % self.n_heads != 0:
            raise ArgumentError(N.FB2_INVALID_ARG,
                                f"DModel ({self.d_model}) must be divisible by NHeads ({self.n_heads}).")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def mlp_hidden(self) -> int:
        return 4 * self.d_model


def param_names(cfg: ModelConfig) -> list[str]:
    """Parameters.Names in registration order (GptModel.cs:14-18, 47-98)."""
    block = ["ln1.w", "ln1.b", "attn.qkv.w", "attn.qkv.b", "attn.proj.w", "attn.proj.b",
             "ln2.w", "ln2.b", "mlp.fc.w", "mlp.fc.b", "mlp.proj.w", "mlp.proj.b"]
    names = ["tok_emb", "pos_emb"]
    for i in range(cfg.n_layers):
        names += [f"blocks.{i}.{b}" for b in block]
    return names + ["ln_f.w", "ln_f.b"]


def param_shapes(cfg: ModelConfig) -> list[tuple[int, ...]]:
    D, F = cfg.d_model, cfg.mlp_hidden
    shapes: list[tuple[int, ...]] = [(cfg.vocab_size, D), (cfg.context_length, D)]
    for _ in range(cfg.n_layers):
        shapes += [(D,), (D,), (D, 3 * D), (3 * D,), (D, D), (D,), (D,), (D,), (D, F), (F,), (F, D), (D,)]
    return shapes + [(D,), (D,)]


def init_params(cfg: ModelConfig, seed: int) -> list[np.ndarray]:
    """Seeded synthetic weights: those `new GptModel(cfg, backend,
    new Random(seed))` creates (GptModel.cs:47-98), computed by the library's
    host code (fb2_init_params)."""
    params = [np.empty(s, np.float32) for s in param_shapes(cfg)]
    desc = N.ModelDesc(cfg.vocab_size, cfg.context_length, cfg.d_model, cfg.n_layers, cfg.n_heads,
                       N.FB2_WEIGHTS_FP32)
    ptrs = (C.c_void_p * len(params))(*[a.ctypes.data for a in params])
    N.check(N.load().fb2_init_params(C.byref(desc), int(seed), ptrs, len(params)))
    return params


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _dtype_code(weight_dtype: str) -> int:
    if weight_dtype not in ("fp32", "bf16"):
        raise ArgumentError(N.FB2_INVALID_ARG, "weight_dtype must be 'fp32' or 'bf16'")
    return N.FB2_WEIGHTS_BF16 if weight_dtype == "bf16" else N.FB2_WEIGHTS_FP32


def read_forgemodel_header(path: str) -> tuple[ModelConfig, str]:
    """Validate a FORGEMODEL1 checkpoint (every rule of Checkpoint.LoadCore,
    Checkpoint.cs:174-264, checksum included) and return its configuration
    and ModelName.  No device needed."""
    desc = N.ModelDesc()
    name = C.create_string_buffer(4096)
    N.check(N.load().fb2_forgemodel_read_header(str(path).encode(), C.byref(desc), name, len(name)))
    return (ModelConfig(desc.vocab_size, desc.context_length, desc.d_model, desc.n_layers, desc.n_heads),
            name.value.decode("utf-8"))


def write_forgemodel(path: str, cfg: ModelConfig, params: Sequence[np.ndarray], model_name: str) -> None:
    """Write a FORGEMODEL1 model checkpoint (Checkpoint.SaveTraining's layout,
    Checkpoint.cs:63-119, 143-166, with no optimizer state)."""
    shapes = param_shapes(cfg)
    if len(params) != len(shapes):
        raise ArgumentError(N.FB2_INVALID_ARG, f"expected {len(shapes)} parameter tensors, got {len(params)}")
    arrs = [np.ascontiguousarray(p, dtype=np.float32) for p in params]
    for a, s in zip(arrs, shapes):
        if a.size != int(np.prod(s)):
            raise ArgumentError(N.FB2_INVALID_ARG, f"parameter of shape {a.shape} does not match {s}")
    desc = N.ModelDesc(cfg.vocab_size, cfg.context_length, cfg.d_model, cfg.n_layers, cfg.n_heads,
                       N.FB2_WEIGHTS_FP32)
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    N.check(N.load().fb2_forgemodel_write(str(path).encode(), C.byref(desc), model_name.encode("utf-8"), ptrs,
                                          len(arrs)))


def _ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data) if a is not None and a.size else None


class B200Backend:
    """`--backend b200`: fp32 weights resident on one or more B200s plus a
    decode session (KV caches, histories, RNG streams, decode-step graphs).

    params: the model's weights in Parameters.Names order (float32 arrays of
    the shapes `param_shapes(config)` gives), e.g. as Checkpoint.LoadCore
    read them (src/LLM.Core/Checkpoint/Checkpoint.cs:222-227).  The library
    copies them; the caller keeps ownership.  weight_dtype "bf16" stores
    tok_emb and the projections rounded to bf16 (FB2_WEIGHTS_BF16).
    """

    def __init__(self, config: ModelConfig, params: Sequence[np.ndarray], devices: Iterable[int] | None = None,
                 max_seqs: int = 1, weight_dtype: str = "fp32"):
        if weight_dtype not in ("fp32", "bf16"):
            raise ArgumentError(N.FB2_INVALID_ARG, "weight_dtype must be 'fp32' or 'bf16'")
        self.config = config
        L = N.load()
        shapes = param_shapes(config)
        if len(params) != len(shapes):
            raise ArgumentError(N.FB2_INVALID_ARG, f"expected {len(shapes)} parameter tensors, got {len(params)}")
        self._params = []
        for p, s in zip(params, shapes):
            a = np.ascontiguousarray(p, dtype=np.float32)
            if a.size != int(np.prod(s)):
                raise ArgumentError(N.FB2_INVALID_ARG, f"parameter of shape {a.shape} does not match {s}")
            self._params.append(a)
        desc = N.ModelDesc(config.vocab_size, config.context_length, config.d_model, config.n_layers,
                           config.n_heads, _dtype_code(weight_dtype))
        ptrs = (C.c_void_p * len(self._params))(*[a.ctypes.data for a in self._params])
        devs = _i32(list(devices) if devices is not None else [0])
        self._model = C.c_void_p()
        N.check(L.fb2_model_create(C.byref(desc), ptrs, len(self._params), _ptr(devs), len(devs),
                                   C.byref(self._model)))
        self._params = None  # the device copies are authoritative now
        self._open_session(devs, max_seqs)

    @classmethod
    def from_forgemodel(cls, path: str, devices: Iterable[int] | None = None, max_seqs: int = 1,
                        weight_dtype: str = "fp32") -> "B200Backend":
        """Checkpoint.Load (src/LLM.Core/Checkpoint/Checkpoint.cs:121-122)
        straight to the devices: the library validates the FORGEMODEL1 file
        (header rules, registry names, payload size, SHA-256) and uploads it;
        InvalidDataError where the reference throws InvalidDataException."""
        self = cls.__new__(cls)
        L = N.load()
        devs = _i32(list(devices) if devices is not None else [0])
        desc = N.ModelDesc()
        self._model = C.c_void_p()
        N.check(L.fb2_model_load_forgemodel(str(path).encode(), _dtype_code(weight_dtype), _ptr(devs), len(devs),
                                            C.byref(desc), C.byref(self._model)))
        self.config = ModelConfig(desc.vocab_size, desc.context_length, desc.d_model, desc.n_layers, desc.n_heads)
        self._params = None
        self._open_session(devs, max_seqs)
        return self

    def _open_session(self, devs: np.ndarray, max_seqs: int) -> None:
        L = N.load()
        self.max_seqs = int(max_seqs)
        self._session = C.c_void_p()
        try:
            N.check(L.fb2_session_create(self._model, self.max_seqs, C.byref(self._session)))
        except Exception:
            L.fb2_model_destroy(self._model)
            self._model = None
            raise
        self.devices = [int(d) for d in devs]

    # -- lifetime -------------------------------------------------------------
    def close(self) -> None:
        L = N.load()
        if getattr(self, "_session", None):
            L.fb2_session_destroy(self._session)
            self._session = None
        if getattr(self, "_model", None):
            L.fb2_model_destroy(self._model)
            self._model = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- configuration --------------------------------------------------------
    def set_stream(self, cuda_stream: int | None, device_slot: int = 0) -> None:
        """Runs this backend's work on the caller's CUDA stream (e.g.
        torch.cuda.current_stream().cuda_stream); None restores its own."""
        N.check(N.load().fb2_session_set_stream(self._session, device_slot,
                                                C.c_void_p(cuda_stream) if cuda_stream else None))

    def seed(self, slot: int, seed: int) -> None:
        N.check(N.load().fb2_session_seed(self._session, slot, seed))

    # -- GptModel.ForwardLast ---------------------------------------------------
    def forward_last(self, tokens: Sequence[int]) -> np.ndarray:
        """Logits [V] of the last position (GptModel.cs:202-209)."""
        return self.forward_last_batch([tokens])[0]

    def forward_last_batch(self, windows: Sequence[Sequence[int]]) -> np.ndarray:
        lens = _i32([len(w) for w in windows])
        toks = _i32(np.concatenate([np.asarray(w, np.int64) for w in windows]) if len(windows) else [])
        out = np.empty((len(windows), self.config.vocab_size), np.float32)
        N.check(N.load().fb2_forward_last_logits(self._session, len(windows), _ptr(toks), _ptr(lens), _ptr(out)))
        return out

    def teacher_forced_logits(self, tokens: np.ndarray, prompt_len: int) -> np.ndarray:
        """Prefill tokens[:, :prompt_len], then feed the rest one at a time
        through the KV-cached decode step; logits after every prefix length
        prompt_len..len: [n, len - prompt_len + 1, V]."""
        t = _i32(tokens)
        if t.ndim != 2:
            raise ArgumentError(N.FB2_INVALID_ARG, "tokens must be [n_seqs, len]")
        n, ln = t.shape
        out = np.empty((n, ln - prompt_len + 1, self.config.vocab_size), np.float32)
        N.check(N.load().fb2_teacher_forced_logits(self._session, n, _ptr(t), ln, prompt_len, _ptr(out)))
        return out

    # -- Sampler ----------------------------------------------------------------
    @staticmethod
    def _sampling(max_new: int, temperature: float, top_k: int, eos_id, penalty: float, ngram: int):
        return N.Sampling(float(temperature), int(top_k), float(penalty), int(ngram),
                          -1 if eos_id is None else int(eos_id), int(max_new))

    def sample_logits(self, logits: np.ndarray, windows: Sequence[Sequence[int]], temperature: float, top_k: int,
                      uniforms: Sequence[float] | None, repetition_penalty: float = 1.0,
                      no_repeat_ngram_size: int = 0) -> np.ndarray:
        """ApplyRepetitionControls + Sample (Sampler.cs:29-69, 96-104,
        111-165) on the device for each logit row; uniforms[i] is row i's
        NextDouble() value."""
        lg = np.ascontiguousarray(logits, np.float32)
        if lg.ndim == 1:
            lg = lg[None, :]
        n = lg.shape[0]
        if lg.shape[1] != self.config.vocab_size:
            raise ArgumentError(N.FB2_INVALID_ARG, "logit rows must have vocab_size entries")
        wl = _i32([len(w) for w in windows])
        wt = _i32(np.concatenate([np.asarray(w, np.int64) for w in windows]) if wl.sum() else [0])
        u = np.ascontiguousarray(uniforms, np.float64) if uniforms is not None else None
        sp = self._sampling(1, temperature, top_k, None, repetition_penalty, no_repeat_ngram_size)
        out = np.empty(n, np.int32)
        N.check(N.load().fb2_sample_logits(self._session, n, _ptr(lg), _ptr(wt), _ptr(wl), C.byref(sp),
                                           _ptr(u) if u is not None else None, _ptr(out)))
        return out

    def generate_batch(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, temperature: float, top_k: int,
                       rng: DotNetRandom | Sequence[DotNetRandom] | None = None, eos_id: int | None = None,
                       repetition_penalty: float = 1.0, no_repeat_ngram_size: int = 0,
                       seeds: Sequence[int] | None = None, uniforms: np.ndarray | None = None,
                       on_token: Callable[[int, int, int], bool | None] | None = None) -> list[np.ndarray]:
        """Sampler.Generate for independent sequences (one window each).

        Uniform source, in order of precedence: `uniforms` [n, max_new];
        `seeds` (a fresh `new Random(seed)` per sequence); `rng` (one
        DotNetRandom per sequence, or one shared by all: the library pulls
        each value from it through FB2_RNG_CALLBACK when it samples, so the
        generator advances by exactly the draws the reference makes)."""
        n = len(prompts)
        if n == 0:
            return []
        if max_new_tokens < 0:
            raise ArgumentError(N.FB2_INVALID_ARG, "maxNewTokens must be >= 0.")
        lens = _i32([len(p) for p in prompts])
        if (lens <= 0).any():
            raise ArgumentError(N.FB2_INVALID_ARG, "Need at least one prompt token.")
        toks = _i32(np.concatenate([np.asarray(p, np.int64) for p in prompts]))
        sp = self._sampling(max_new_tokens, temperature, top_k, eos_id, repetition_penalty, no_repeat_ngram_size)
        mode, seed_arr, uni = N.FB2_RNG_UNIFORMS, None, None
        rngs = None
        if uniforms is not None:
            uni = np.ascontiguousarray(uniforms, np.float64).reshape(n, max(max_new_tokens, 1))
        elif seeds is not None:
            mode, seed_arr = N.FB2_RNG_SEEDS, _i32(seeds)
        elif rng is not None:
            rngs = [rng] * n if isinstance(rng, DotNetRandom) else list(rng)
            if len(rngs) != n:
                raise ArgumentError(N.FB2_INVALID_ARG, "one rng per sequence")
            mode = N.FB2_RNG_CALLBACK
        elif temperature > 0:
            raise ArgumentError(N.FB2_INVALID_ARG, "rng is required when temperature > 0")
        out = np.zeros((n, max(max_new_tokens, 1)), np.int32)
        counts = np.zeros(n, np.int32)
        cb = N.TOKEN_CB(0)
        if on_token is not None:
            def _cb(user, seq, step, token):
                r = on_token(seq, step, token)
                return 1 if r else 0
            cb = N.TOKEN_CB(_cb)
        L = N.load()
        ucb = N.UNIFORM_CB(0)
        if rngs is not None:
            ucb = N.UNIFORM_CB(lambda user, seq: rngs[seq].next_double())
        N.check(L.fb2_session_set_uniform_source(self._session, ucb, None))
        try:
            N.check(L.fb2_generate(self._session, n, _ptr(toks), _ptr(lens), C.byref(sp), mode,
                                   _ptr(seed_arr) if seed_arr is not None else None,
                                   _ptr(uni) if uni is not None else None, _ptr(out), _ptr(counts), cb, None))
        finally:
            L.fb2_session_set_uniform_source(self._session, N.UNIFORM_CB(0), None)
        return [out[i, :counts[i]].copy() for i in range(n)]

    def generate(self, prompt_tokens: Sequence[int], max_new_tokens: int, temperature: float, top_k: int,
                 rng: DotNetRandom | None, eos_id: int | None = None, repetition_penalty: float = 1.0,
                 no_repeat_ngram_size: int = 0) -> list[int]:
        """Sampler.Generate (Sampler.cs:78-109) for one sequence."""
        if rng is None and temperature > 0:
            raise ArgumentError(N.FB2_INVALID_ARG, "rng must not be null")
        return self.generate_batch([prompt_tokens], max_new_tokens, temperature, top_k,
                                   rng=[rng] if rng is not None else None, eos_id=eos_id,
                                   repetition_penalty=repetition_penalty,
                                   no_repeat_ngram_size=no_repeat_ngram_size)[0].tolist()

    def generate_device(self, prompt_tokens_ptr: int, prompt_lens_ptr: int, prompt_lens: Sequence[int],
                        max_new_tokens: int, temperature: float, top_k: int, out_tokens_ptr: int,
                        out_counts_ptr: int, eos_id: int | None = None, repetition_penalty: float = 1.0,
                        no_repeat_ngram_size: int = 0, seeds: Sequence[int] | None = None,
                        uniforms_ptr: int | None = None) -> None:
        """fb2_generate_device: inputs/outputs already on the device (raw
        pointers, e.g. torch tensors' data_ptr()); returns once enqueued."""
        sp = self._sampling(max_new_tokens, temperature, top_k, eos_id, repetition_penalty, no_repeat_ngram_size)
        hl = _i32(prompt_lens)
        mode = N.FB2_RNG_UNIFORMS if uniforms_ptr else N.FB2_RNG_SEEDS
        sa = _i32(seeds) if seeds is not None else None
        N.check(N.load().fb2_generate_device(self._session, len(hl), C.c_void_p(prompt_tokens_ptr),
                                             C.c_void_p(prompt_lens_ptr), _ptr(hl), C.byref(sp), mode,
                                             _ptr(sa) if sa is not None else None,
                                             C.c_void_p(uniforms_ptr) if uniforms_ptr else None,
                                             C.c_void_p(out_tokens_ptr), C.c_void_p(out_counts_ptr)))

    def stats(self) -> dict:
        s = N.Stats()
        N.check(N.load().fb2_stats(self._session, C.byref(s)))
        return {k: getattr(s, k) for k, _ in N.Stats._fields_ if k != "reserved"}

    def reset_stats(self) -> None:
        N.check(N.load().fb2_stats_reset(self._session))


class Sampler:
    """Static entry points shaped like src/LLM.Core/Inference/Sampler.cs."""

    @staticmethod
    def generate(model: B200Backend, prompt_tokens: Sequence[int], max_new_tokens: int, temperature: float,
                 top_k: int, rng: DotNetRandom | None, eos_id: int | None = None, repetition_penalty: float = 1.0,
                 no_repeat_ngram_size: int = 0) -> list[int]:
        if model is None:
            raise ArgumentError(N.FB2_INVALID_ARG, "model must not be null")
        if prompt_tokens is None or len(prompt_tokens) == 0:
            raise ArgumentError(N.FB2_INVALID_ARG, "Need at least one prompt token.")
        return model.generate(prompt_tokens, max_new_tokens, temperature, top_k, rng, eos_id, repetition_penalty,
                              no_repeat_ngram_size)

    @staticmethod
    def sample(model: B200Backend, logits: np.ndarray, temperature: float, top_k: int, rng: DotNetRandom) -> int:
        """Sampler.Sample (Sampler.cs:29-69) on the device."""
        lg = np.ascontiguousarray(logits, np.float32)
        if lg.size == 0:
            raise ArgumentError(N.FB2_INVALID_ARG, "Need at least one logit.")
        if not np.isfinite(temperature):
            raise ArgumentError(N.FB2_INVALID_ARG, "Temperature must be finite.")
        u = [rng.next_double()] if temperature > 0 else None
        return int(model.sample_logits(lg, [[]], temperature, top_k, u)[0])


class BpeTokenizer:
    """The byte-level BPE tokenizer (src/LLM.Core/Tokenizer/BpeTokenizer.cs)
    in the library: load (BpeTokenizer.Load's checks; InvalidDataError where
    it throws InvalidDataException), Encode, EncodeDocument, Decode, and a
    UTF-8 stream decoder for tokens printed as they are generated."""

    def __init__(self, path: str):
        self._t = C.c_void_p()
        N.check(N.load().fb2_tokenizer_load(str(path).encode(), C.byref(self._t)))
        vs, eos = C.c_int32(), C.c_int32()
        N.check(N.load().fb2_tokenizer_info(self._t, C.byref(vs), C.byref(eos)))
        self.vocab_size, self.eos_token_id = vs.value, eos.value

    def close(self) -> None:
        if getattr(self, "_t", None):
            N.load().fb2_tokenizer_destroy(self._t)
            self._t = None

    def __del__(self):
        self.close()

    def encode(self, data: str | bytes) -> list[int]:
        b = data.encode("utf-8") if isinstance(data, str) else bytes(data)
        buf = np.frombuffer(b, np.uint8) if b else np.zeros(1, np.uint8)
        out = np.empty(max(len(b), 1), np.int32)
        n = C.c_int64()
        N.check(N.load().fb2_tokenizer_encode(self._t, buf.ctypes.data, len(b), out.ctypes.data, out.size,
                                              C.byref(n)))
        return out[:n.value].tolist()

    def encode_document(self, data: str | bytes) -> list[int]:
        """EncodeDocument (BpeTokenizer.cs:244-251): the text, then EOS."""
        return self.encode(data) + [self.eos_token_id]

    def decode_bytes(self, ids: Sequence[int]) -> bytes:
        a = _i32(list(ids)) if len(ids) else np.zeros(1, np.int32)
        n = C.c_int64()
        L = N.load()
        st = L.fb2_tokenizer_decode(self._t, a.ctypes.data, len(ids), None, 0, C.byref(n))
        if st != N.FB2_OK and n.value == 0:
            N.check(st)
        out = np.empty(max(n.value, 1), np.uint8)
        N.check(L.fb2_tokenizer_decode(self._t, a.ctypes.data, len(ids), out.ctypes.data, out.size, C.byref(n)))
        return out[:n.value].tobytes()

    def decode(self, ids: Sequence[int]) -> str:
        """Decode (BpeTokenizer.cs:320-339): UTF-8 with replacement characters."""
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def stream_decoder(self):
        """Utf8StreamDecoder (BpeTokenizer.cs:57-78): keeps incomplete UTF-8
        sequences until later tokens complete them."""
        import codecs
        dec = codecs.getincrementaldecoder("utf-8")("replace")
        tok = self

        class _Stream:
            def decode_token(self, token_id: int) -> str:
                return dec.decode(tok.decode_bytes([token_id]))

            def flush(self) -> str:
                return dec.decode(b"", final=True)

        return _Stream()
