"""ctypes bindings of libforge_b200.so (include/forge_b200.h).

The product path: every call goes to the CUDA library.  There is no CPU
fallback; if the library or a CUDA device is missing, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libforge_b200.so")

FB2_OK = 0
FB2_INVALID_ARG = -1
FB2_OUT_OF_MEMORY = -2
FB2_CUDA_ERROR = -3
FB2_TIMEOUT = -4
FB2_UNSUPPORTED = -5
FB2_NO_DEVICE = -6
FB2_INVALID_DATA = -7

FB2_WEIGHTS_FP32 = 0
FB2_WEIGHTS_BF16 = 1

FB2_RNG_SEEDS = 0
FB2_RNG_SESSION = 1
FB2_RNG_UNIFORMS = 2
FB2_RNG_CALLBACK = 3

# Every symbol include/forge_b200.h declares.
EXPORTED = [
    "fb2_version", "fb2_last_error", "fb2_device_count", "fb2_model_create", "fb2_model_destroy",
    "fb2_session_create", "fb2_session_destroy", "fb2_session_seed", "fb2_session_set_uniform_source",
    "fb2_session_set_stream",
    "fb2_generate", "fb2_generate_device", "fb2_forward_last_logits", "fb2_teacher_forced_logits",
    "fb2_sample_logits", "fb2_forward_last_logits_noalloc", "fb2_init_params", "fb2_stats", "fb2_stats_reset",
    "fb2_forgemodel_read_header", "fb2_model_load_forgemodel", "fb2_forgemodel_write",
    "fb2_tokenizer_load", "fb2_tokenizer_destroy", "fb2_tokenizer_info", "fb2_tokenizer_encode",
    "fb2_tokenizer_decode",
]
TEST_EXPORTED = ["fb2_test_expf", "fb2_test_expf_hash", "fb2_test_dotnet_random", "fb2_test_mk_trace",
                 "fb2_test_gemm_tc", "fb2_test_sha256", "fb2_test_mk_withhold", "fb2_test_fail_alloc", "fb2_test_mk_geometry"]


class ModelDesc(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("context_length", C.c_int32), ("d_model", C.c_int32),
                ("n_layers", C.c_int32), ("n_heads", C.c_int32), ("weight_dtype", C.c_int32)]


class Sampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("repetition_penalty", C.c_float),
                ("no_repeat_ngram", C.c_int32), ("eos_id", C.c_int32), ("max_new_tokens", C.c_int32)]


class Stats(C.Structure):
    _fields_ = [("tokens_generated", C.c_int64), ("decode_steps", C.c_int64), ("prefill_rows", C.c_int64),
                ("reprefills", C.c_int64), ("prefill_ms", C.c_double), ("decode_ms", C.c_double),
                ("sample_ms", C.c_double), ("kernel_launches", C.c_int64), ("device_count", C.c_int32),
                ("reserved", C.c_int32), ("persistent_steps", C.c_int64), ("reused_prefix_rows", C.c_int64)]


TOKEN_CB = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_int32)
UNIFORM_CB = C.CFUNCTYPE(C.c_double, C.c_void_p, C.c_int32)

_lib = None


class NativeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


class ArgumentError(ValueError, NativeError):
    """INVALID_ARG: the reference throws ArgumentException / ArgumentOutOfRangeException."""


class InvalidDataError(NativeError):
    """INVALID_DATA: a checkpoint the reference rejects with InvalidDataException
    (Checkpoint.cs:174-264)."""


def load(path: str | None = None):
    """Loads the CUDA library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise OSError(f"libforge_b200.so not built at {p}; run __graft_entry__.build()")
    L = C.CDLL(p)
    vp, i32, i64, f32p, i32p, f64p = C.c_void_p, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p
    L.fb2_version.restype = i32
    L.fb2_last_error.restype = C.c_char_p
    L.fb2_device_count.argtypes = [C.POINTER(i32)]
    L.fb2_model_create.argtypes = [C.POINTER(ModelDesc), C.POINTER(vp), i32, i32p, i32, C.POINTER(vp)]
    L.fb2_model_destroy.argtypes = [vp]
    L.fb2_model_destroy.restype = None
    L.fb2_session_create.argtypes = [vp, i32, C.POINTER(vp)]
    L.fb2_session_destroy.argtypes = [vp]
    L.fb2_session_destroy.restype = None
    L.fb2_session_seed.argtypes = [vp, i32, i32]
    L.fb2_session_set_stream.argtypes = [vp, i32, vp]
    L.fb2_session_set_uniform_source.argtypes = [vp, UNIFORM_CB, vp]
    L.fb2_generate.argtypes = [vp, i32, i32p, i32p, C.POINTER(Sampling), i32, i32p, f64p, i32p, i32p, TOKEN_CB, vp]
    L.fb2_generate_device.argtypes = [vp, i32, vp, vp, i32p, C.POINTER(Sampling), i32, i32p, vp, vp, vp]
    L.fb2_forward_last_logits.argtypes = [vp, i32, i32p, i32p, f32p]
    L.fb2_teacher_forced_logits.argtypes = [vp, i32, i32p, i32, i32, f32p]
    L.fb2_sample_logits.argtypes = [vp, i32, f32p, i32p, i32p, C.POINTER(Sampling), f64p, i32p]
    L.fb2_init_params.argtypes = [C.POINTER(ModelDesc), i32, C.POINTER(vp), i32]
    L.fb2_forward_last_logits_noalloc.argtypes = [vp, i32, i32, vp, vp, vp]
    L.fb2_stats.argtypes = [vp, C.POINTER(Stats)]
    L.fb2_stats_reset.argtypes = [vp]
    L.fb2_test_expf.argtypes = [f32p, f32p, i64]
    L.fb2_test_expf_hash.argtypes = [C.c_uint32, i32, vp]
    L.fb2_test_dotnet_random.argtypes = [i32, i32, vp]
    L.fb2_test_mk_trace.argtypes = [vp, vp, i64, C.POINTER(i32), C.POINTER(i32)]
    L.fb2_test_gemm_tc.argtypes = [i32, i32, i32, vp, vp, vp]
    L.fb2_test_sha256.argtypes = [vp, i64, vp]
    L.fb2_test_mk_withhold.argtypes = [vp, i32, i64]
    L.fb2_test_fail_alloc.argtypes = [i64, C.POINTER(i64)]
    L.fb2_test_mk_geometry.argtypes = [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]
    L.fb2_forgemodel_read_header.argtypes = [C.c_char_p, C.POINTER(ModelDesc), C.c_char_p, i32]
    L.fb2_model_load_forgemodel.argtypes = [C.c_char_p, i32, i32p, i32, C.POINTER(ModelDesc), C.POINTER(vp)]
    L.fb2_forgemodel_write.argtypes = [C.c_char_p, C.POINTER(ModelDesc), C.c_char_p, C.POINTER(vp), i32]
    L.fb2_tokenizer_load.argtypes = [C.c_char_p, C.POINTER(vp)]
    L.fb2_tokenizer_destroy.argtypes = [vp]
    L.fb2_tokenizer_destroy.restype = None
    L.fb2_tokenizer_info.argtypes = [vp, C.POINTER(i32), C.POINTER(i32)]
    L.fb2_tokenizer_encode.argtypes = [vp, vp, i64, vp, i64, C.POINTER(i64)]
    L.fb2_tokenizer_decode.argtypes = [vp, vp, i64, vp, i64, C.POINTER(i64)]
    for name in EXPORTED + TEST_EXPORTED:
        fn = getattr(L, name)
        if fn.restype is C.c_int:  # default
            fn.restype = i32
    _lib = L
    return L


def check(status: int) -> None:
    if status == FB2_OK:
        return
    msg = (load().fb2_last_error() or b"").decode(errors="replace")
    if status == FB2_INVALID_ARG:
        raise ArgumentError(status, msg)
    if status == FB2_INVALID_DATA:
        raise InvalidDataError(status, msg)
    raise NativeError(status, msg)
