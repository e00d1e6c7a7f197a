"""C-ABI library checks that need no GPU: it loads, exports every symbol the
headers declare, and rejects bad arguments with status codes (never aborts)."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(fb2_[a-z0-9_]+)\s*\(", text):
            syms.add(m.group(1))
    return syms


def test_library_exports_every_declared_symbol(pkg):
    from forge_lm_b200 import _native as N
    L = N.load()
    declared = _declared_symbols()
    assert "fb2_generate" in declared and "fb2_model_create" in declared
    for s in declared:
        assert hasattr(L, s), f"libforge_b200.so does not export {s}"
    assert set(N.EXPORTED) | set(N.TEST_EXPORTED) >= declared


def test_version_and_errors_without_device(pkg):
    from forge_lm_b200 import _native as N
    L = N.load()
    assert L.fb2_version() == 1
    n = C.c_int32(-1)
    assert L.fb2_device_count(C.byref(n)) == N.FB2_OK and n.value >= 0
    assert L.fb2_device_count(None) == N.FB2_INVALID_ARG
    assert b"NULL" in L.fb2_last_error()
    out = C.c_void_p()
    assert L.fb2_model_create(None, None, 0, None, 0, C.byref(out)) == N.FB2_INVALID_ARG
    # inconsistent config is rejected before any device work
    desc = N.ModelDesc(32, 8, 15, 2, 2, 0)
    arr = np.zeros(1, np.float32)
    ptrs = (C.c_void_p * 28)(*([arr.ctypes.data] * 28))
    assert L.fb2_model_create(C.byref(desc), ptrs, 28, None, 0, C.byref(out)) == N.FB2_INVALID_ARG
    assert b"divisible" in L.fb2_last_error()
    assert L.fb2_session_create(None, 1, C.byref(out)) == N.FB2_INVALID_ARG
    assert L.fb2_generate(None, 1, None, None, None, 0, None, None, None, None, N.TOKEN_CB(0), None) == \
        N.FB2_INVALID_ARG
    assert L.fb2_stats(None, None) == N.FB2_INVALID_ARG


def test_model_config_validation(pkg):
    with pytest.raises(ValueError):
        pkg.ModelConfig(32, 8, 15, 2, 2)
    with pytest.raises(ValueError):
        pkg.ModelConfig(0, 8, 16, 2, 2)
    cfg = pkg.ModelConfig(32, 8, 16, 2, 2)
    assert cfg.head_dim == 8 and cfg.mlp_hidden == 64
    assert sum(int(np.prod(s)) for s in pkg.param_shapes(cfg)) == 7232
    assert pkg.param_names(cfg)[:3] == ["tok_emb", "pos_emb", "blocks.0.ln1.w"]
    assert pkg.param_names(cfg)[-2:] == ["ln_f.w", "ln_f.b"]


def test_param_names_match_oracle(pkg, O):
    cfg = pkg.ModelConfig(40, 10, 16, 3, 2)
    assert pkg.param_names(cfg) == O.param_names(O.Config(40, 10, 16, 3, 2))


@pytest.mark.skipif(os.environ.get("FORGE_B200_HAVE_GPU") == "1", reason="host without a CUDA device only")
def test_backend_fails_loudly_without_device(pkg, O):
    """No CPU fallback: without a CUDA device the backend raises."""
    if pkg.device_count() > 0:
        pytest.skip("a CUDA device is present")
    cfg = pkg.ModelConfig(32, 8, 16, 2, 2)
    params = O.init_params(O.Config(32, 8, 16, 2, 2), 1)
    with pytest.raises(pkg.NativeError):
        pkg.B200Backend(cfg, params)


def test_expf_fixup_table_matches_host_libm(O):
    """The generated table lists exactly the inputs where the host expf
    differs from (float)exp((double)x) (spot-checked on a sample)."""
    path = os.path.join(ROOT, "forge-lm_b200", "csrc", "generated", "expf_fixups.inc")
    assert os.path.exists(path)
    pairs = []
    with open(path) as f:
        for line in f:
            if line.startswith("0x"):
                a, b = line.strip().rstrip(",").split(",")
                pairs.append((int(a.rstrip("u"), 16), int(b.rstrip("u"), 16)))
    assert len(pairs) > 1000
    ins = np.array([p[0] for p in pairs], np.uint32)
    assert np.all(np.diff(ins.astype(np.int64)) > 0)  # sorted for the device binary search
    sel = np.random.default_rng(0).choice(len(pairs), 2000, replace=False)
    x = ins[sel].view(np.float32)
    assert np.array_equal(O.expf(x).view(np.uint32), np.array([pairs[i][1] for i in sel], np.uint32))
    # a range scan on the host agrees with the table's entries in that range
    lo, hi = 0xBF000000, 0xBF0FFFFF
    n, bad = O.expf_vs_double_scan(lo, hi, 1 << 16)
    in_range = ins[(ins >= lo) & (ins <= hi)]
    assert n == len(in_range) and np.array_equal(np.sort(bad), in_range)


def test_expf_fixup_midpoint_bound():
    """Every listed input with a normal result has exp(x) within
    FB2_EXPF_FIXUP_MAX_GAP ulp of a rounding midpoint: the device skips the
    table for inputs farther than twice that, so the bound must cover all."""
    path = os.path.join(ROOT, "forge-lm_b200", "csrc", "generated", "expf_fixups.inc")
    txt = open(path).read()
    gap = float(txt.split("#define FB2_EXPF_FIXUP_MAX_GAP")[1].split()[0])
    assert 0.0 < gap < 0.01  # the host expf is within about half an ulp
    body = txt[txt.index("kExpfFixupData[] = {"):txt.index("};")]
    words = np.array([int(w.rstrip("u"), 16) for w in body.replace(",", " ").split() if w.startswith("0x")], np.uint64)
    x = words[0::2].astype(np.uint32).view(np.float32).astype(np.float64)
    e = np.exp(x)
    r = e.astype(np.float32)
    normal = (r >= np.float32(1.17549435e-38)) & (r < np.finfo(np.float32).max)
    rd, en = r[normal].astype(np.float64), e[normal]
    up = np.nextafter(r[normal], np.float32(np.inf)).astype(np.float64) - rd
    dn = rd - np.nextafter(r[normal], np.float32(0)).astype(np.float64)
    g = np.minimum((rd + 0.5 * up - en) / up, (en - (rd - 0.5 * dn)) / dn)
    # numpy's exp and the C runtime's exp may differ by a few double ulps,
    # about 1e-8 float ulps here; the device compares against twice the bound
    assert len(g) > 1000 and g.max() <= gap + 1e-7


def test_library_init_params_equal_oracle(pkg, O):
    """fb2_init_params reproduces GptModel's seeded init bit for bit (the
    same restatement the oracle makes)."""
    for shape, seed in (((32, 8, 16, 2, 2), 42), ((300, 24, 32, 3, 4), 1234)):
        a = pkg.init_params(pkg.ModelConfig(*shape), seed)
        b = O.init_params(O.Config(*shape), seed)
        assert all(np.array_equal(x, y) for x, y in zip(a, b))
