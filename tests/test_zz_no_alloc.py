"""fb2_forward_last_logits_noalloc: the entry point for callers that cannot
call cudaMalloc (under a host runtime that owns the device memory budget,
or on a path that must not synchronise the device).

It must give what the allocating entry point fb2_forward_last_logits gives
(same tolerance as every logits test: max |a-e| / max(1, |e|) <= 1e-3), on
two calls in a row (the shared scratch keeps the previous call's contents),
without taking device memory, and must reject windows beyond its limit.
This file is collected last, and it builds its own model so that it passes
alone in a fresh process as well as after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3
SHAPE = (2256, 256, 256, 4, 4)  # BASELINE configs[0] model shape


def _relerr(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.max(np.abs(a - e) / np.maximum(1.0, np.abs(e))))


@pytest.mark.parametrize("weight_dtype", ["fp32", "bf16"])
def test_noalloc_matches_allocating_entry_point(pkg, weight_dtype):
    """fp32 weights, and bf16 weights (the gemv path that reads 2-byte copies)."""
    import torch
    from forge_lm_b200 import _native as N

    cfg = pkg.ModelConfig(*SHAPE)
    params = pkg.init_params(cfg, 1234)
    be = pkg.B200Backend(cfg, params, devices=[0], weight_dtype=weight_dtype)
    L = N.load()
    try:
        rng = np.random.default_rng(5)
        windows = [rng.integers(0, SHAPE[0], n).astype(np.int32) for n in (12, 16)]
        stream = torch.cuda.Stream(device=0)
        d_logits = torch.empty(SHAPE[0], dtype=torch.float32, device="cuda:0")
        ncall = 0
        for w in windows:
            want = be.forward_last(w)  # the allocating entry point
            d_tok = torch.from_numpy(w).to("cuda:0")
            for call in range(2):  # two calls in a row on the shared scratch
                d_logits.fill_(float("nan"))
                torch.cuda.synchronize()
                free_before = torch.cuda.mem_get_info(0)[0]
                N.check(L.fb2_forward_last_logits_noalloc(be._model, 0, len(w), C.c_void_p(d_tok.data_ptr()),
                                                          C.c_void_p(d_logits.data_ptr()),
                                                          C.c_void_p(stream.cuda_stream)))
                stream.synchronize()
                free_after = torch.cuda.mem_get_info(0)[0]
                if ncall > 0:  # the first call on a device does its one-time set-up
                    assert free_after >= free_before, f"call {ncall} took {free_before - free_after} bytes"
                ncall += 1
                got = d_logits.cpu().numpy()
                assert np.all(np.isfinite(got)), f"call {call}: output not fully written"
                err = _relerr(got, want)
                assert err <= TOL, f"window {len(w)}, call {call}: rel/abs error {err}"
        # beyond the limit: a clear error, nothing launched
        long = torch.zeros(17, dtype=torch.int32, device="cuda:0")
        st = L.fb2_forward_last_logits_noalloc(be._model, 0, 17, C.c_void_p(long.data_ptr()),
                                               C.c_void_p(d_logits.data_ptr()), C.c_void_p(stream.cuda_stream))
        assert st == N.FB2_INVALID_ARG
        assert b"limit of 16" in L.fb2_last_error()
    finally:
        be.close()
