"""Failure detection without faulting a GPU.

The reference fails loudly when a backend cannot start or a device call
fails (src/LLM.Core/Tensor/Cuda/CudaBackend.cs:213; explicit backends are
never swallowed, src/LLM.Core/Tensor/BackendSelection.cs:17-20).  The
library's equivalents:
  - every device wait of the persistent decode kernel is bounded; a wait that
    runs out (here: a word one CTA is told never to publish, and a 50 ms
    limit) ends the launch with FB2_TIMEOUT, and the same session then
    generates correctly;
  - a device allocation that fails (injected on the host, in the second
    device copy of a two-copy model) returns FB2_OUT_OF_MEMORY, frees what
    was allocated, and leaves the device usable.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPE = (2256, 96, 128, 2, 4)


def test_bounded_wait_times_out_and_the_session_recovers(pkg, O):
    from forge_lm_b200 import _native as N
    ocfg = O.Config(*SHAPE)
    params = O.init_params(ocfg, 5)
    prompt = np.random.default_rng(1).integers(0, SHAPE[0], 20).astype(np.int32).tolist()
    want = [int(t) for t in O.generate(ocfg, params, prompt, 12, 0.0, 0, O.DotNetRandom(1))]
    L = N.load()
    with pkg.B200Backend(pkg.ModelConfig(*SHAPE), params, devices=[0]) as be:
        N.check(L.fb2_test_mk_withhold(be._session, 0, 50_000_000))
        with pytest.raises(pkg.NativeError) as e:
            be.generate(prompt, 12, 0.0, 0, None)
        assert e.value.status == N.FB2_TIMEOUT, e.value
        got = be.generate(prompt, 12, 0.0, 0, None)  # same session, hook spent
        assert got == want
        assert be.stats()["persistent_steps"] > 0


def _create(N, L, shape, params, devices):
    desc = N.ModelDesc(*shape, N.FB2_WEIGHTS_FP32)
    ptrs = (C.c_void_p * len(params))(*[p.ctypes.data for p in params])
    devs = np.ascontiguousarray(devices, np.int32)
    model = C.c_void_p()
    st = L.fb2_model_create(C.byref(desc), ptrs, len(params), C.c_void_p(devs.ctypes.data), len(devs),
                            C.byref(model))
    return st, model


def _allocs(N, L):
    n = C.c_int64()
    N.check(L.fb2_test_fail_alloc(0, C.byref(n)))
    return n.value


def test_allocation_failure_on_the_second_device_copy(pkg, O):
    import torch
    from forge_lm_b200 import _native as N
    params = [np.ascontiguousarray(p) for p in O.init_params(O.Config(*SHAPE), 6)]
    L = N.load()
    torch.cuda.synchronize()
    # allocations one device copy of the model makes, and one device's session
    a0 = _allocs(N, L)
    st, m1 = _create(N, L, SHAPE, params, [0])
    N.check(st)
    per_copy = _allocs(N, L) - a0
    s1 = C.c_void_p()
    N.check(L.fb2_session_create(m1, 2, C.byref(s1)))
    per_session = _allocs(N, L) - a0 - per_copy
    L.fb2_session_destroy(s1)
    L.fb2_model_destroy(m1)
    assert per_copy >= 3 and per_session >= 3
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    # Two copies on device 0 stand for a two-device model on a one-GPU box.
    # (1) the second copy's 2nd allocation fails inside fb2_model_create
    N.check(L.fb2_test_fail_alloc(per_copy + 2, None))
    st, m = _create(N, L, SHAPE, params, [0, 0])
    N.check(L.fb2_test_fail_alloc(0, None))
    assert st == N.FB2_OUT_OF_MEMORY and not m.value
    assert b"out of memory" in L.fb2_last_error()
    # (2) a two-copy model is fine; its session fails on the second device
    st, m = _create(N, L, SHAPE, params, [0, 0])
    N.check(st)
    N.check(L.fb2_test_fail_alloc(per_session + 2, None))
    s = C.c_void_p()
    st = L.fb2_session_create(m, 2, C.byref(s))
    N.check(L.fb2_test_fail_alloc(0, None))
    assert st == N.FB2_OUT_OF_MEMORY and not s.value
    L.fb2_model_destroy(m)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] >= free0 - (2 << 20), "device memory leaked by the failed creations"
    # the device is still usable, and a model created now is correct
    ocfg = O.Config(*SHAPE)
    with pkg.B200Backend(pkg.ModelConfig(*SHAPE), params, devices=[0]) as be:
        got = be.forward_last(list(range(1, 30)))
    want = O.forward_last(ocfg, params, list(range(1, 30)))
    assert float(np.max(np.abs(got - want) / np.maximum(1.0, np.abs(want)))) <= 1e-3
