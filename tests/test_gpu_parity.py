"""Parity of the CUDA library (through the C ABI) with the CPU oracle.

Tolerances (from the reference, tests/LLM.Core.Tests/GpuBackendTests.cs:90-101,
601-611): fp32 logits max |a-e| / max(1, |e|) <= 1e-3.  Sampled ids:
bit-exact given the same logits, window and uniforms.  Greedy / sampled id
streams: exact, except that a divergence is accepted only at a near-tie of
the oracle's logits (the two candidates within 1e-4 of each other), the
documented effect of fp32 reduction order.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.max(np.abs(a - e) / np.maximum(1.0, np.abs(e))))


TINY = (12, 6, 8, 1, 2)          # GpuBackendTests.cs:599
SMALL = (32, 8, 16, 2, 2)        # InferenceTests.cs:17
C1 = (2256, 256, 256, 4, 4)


def make(pkg, O, shape, seed, max_seqs=1):
    ocfg = O.Config(*shape)
    params = O.init_params(ocfg, seed)
    be = pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0], max_seqs=max_seqs)
    return ocfg, params, be


# ---------------------------------------------------------------------------
def test_device_expf_equals_host_libm_exhaustive(pkg, O):
    """Every float input: the sampler's device exponential returns the host
    C runtime's expf bits (MathF.Exp, Sampler.cs:57)."""
    import ctypes as C
    from forge_lm_b200 import _native as N
    n = 4096  # 2^32 patterns in chunks of 2^20
    dev = np.zeros(n, np.uint64)
    N.check(N.load().fb2_test_expf_hash(0, n, C.c_void_p(dev.ctypes.data)))
    host = O.expf_hash(0, n)
    bad = np.nonzero(dev != host)[0]
    assert bad.size == 0, f"chunks differing from host expf: {bad[:10]}"


def test_forward_last_tiny_golden(pkg, O, golden):
    g = golden["device_logits_tolerance"]
    ocfg, params, be = make(pkg, O, tuple(g["config"]), g["model_seed"])
    with be:
        got = be.forward_last(g["tokens"])
        want = O.forward(ocfg, params, g["tokens"])[-1]
        assert relerr(got, want) <= g["tolerance"]


@pytest.mark.parametrize("shape,seed", [(SMALL, 1), (C1, 1234)])
def test_forward_last_ragged_batch(pkg, O, shape, seed):
    ocfg, params, be = make(pkg, O, shape, seed, max_seqs=5)
    rng = np.random.default_rng(7)
    ctx = shape[1]
    lens = [1, 3, ctx // 2 + 1, ctx - 1, ctx]
    wins = [rng.integers(0, shape[0], L).astype(np.int32) for L in lens]
    with be:
        got = be.forward_last_batch(wins)
        for i, w in enumerate(wins):
            assert relerr(got[i], O.forward_last(ocfg, params, w)) <= TOL, f"window len {lens[i]}"


def test_teacher_forced_decode_matches_full_forward(pkg, O):
    """The KV-cached decode step equals ForwardLast of each prefix."""
    ocfg, params, be = make(pkg, O, C1, 1234, max_seqs=2)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, C1[0], (2, 80)).astype(np.int32)
    with be:
        got = be.teacher_forced_logits(toks, 32)
    assert got.shape == (2, 49, C1[0])
    for s in range(2):
        for k in range(0, 49, 4):
            want = O.forward_last(ocfg, params, toks[s, :32 + k])
            assert relerr(got[s, k], want) <= TOL, (s, k)


# ---------------------------------------------------------------------------
@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (300, 200, 100), (1024, 768, 768), (256, 3072, 768),
                                   (200, 768, 3072), (17, 768, 768), (64, 2304, 768), (64, 768, 3072),
                                   (100, 36, 100)])
def test_tensor_core_gemm_3xtf32(pkg, M, N, K):
    """The tcgen05 3xTF32 GEMM of the projections against an fp64 product,
    ragged M, N, K: 128-column tiles (M >= 128) and 32-column split-K tiles
    (decode batches, M < 128).  The bound (relative to the largest output) is
    3xTF32 accuracy with the tensor cores' fp32 accumulation, which grows with
    the depth K: 2e-5 up to K = 768, 5e-5 at K = 3072.  A single TF32 product
    would be ~1e-3, the logits tolerance of the parity tests."""
    from forge_lm_b200 import _native as nat
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    out = np.full((M, N), np.nan, np.float32)
    nat.check(nat.load().fb2_test_gemm_tc(M, N, K, A.ctypes.data, W.ctypes.data, out.ctypes.data))
    want = A.astype(np.float64) @ W.astype(np.float64)
    err = float(np.max(np.abs(out - want)) / np.max(np.abs(want)))
    assert err < (2e-5 if K <= 768 else 5e-5), err


def _rows_cases(V, rng):
    cases = []
    for t in range(40):
        lg = (rng.standard_normal(V) * rng.choice([0.5, 2.0, 8.0])).astype(np.float32)
        if t % 5 == 1:  # many ties around the k-th value
            lg = np.round(lg * 2) / 2
        if t % 7 == 2:
            lg[rng.integers(0, V, 20)] = -np.inf
        win = rng.integers(0, V, rng.integers(0, 60)).astype(np.int32)
        if t % 6 == 3 and len(win) > 4:  # repeated n-grams
            win = np.concatenate([win[:4], win[:4], win[:3]]).astype(np.int32)
        cases.append((lg, win))
    return cases


@pytest.mark.parametrize("V", [2256, 16384, 7])
@pytest.mark.parametrize("temperature,top_k,penalty,ngram", [
    (0.0, 0, 1.0, 0), (0.7, 30, 1.1, 4), (1.0, 0, 1.0, 0), (0.8, 40, 1.0, 0), (0.5, 1, 2.0, 1),
    (1.3, 100000, 1.5, 2), (0.9, 5, 1.0, 3)])
def test_sampler_bit_exact(pkg, O, V, temperature, top_k, penalty, ngram):
    shape = (V, 8, 16, 1, 2)
    _, _, be = make(pkg, O, shape, 1)
    rng = np.random.default_rng(V + top_k)
    cases = _rows_cases(V, rng)
    if V == 7:  # all tokens banned -> pre-ban logits restored (Sampler.cs:156-164)
        cases.append((np.arange(7, dtype=np.float32), np.arange(7, dtype=np.int32)))
    logits = np.stack([c[0] for c in cases])
    wins = [c[1] for c in cases]
    uni = rng.random(len(cases))
    with be:
        got = be.sample_logits(logits, wins, temperature, top_k, uni, penalty, ngram)
    for i, (lg, w) in enumerate(cases):
        adj = lg
        if penalty != 1.0 or ngram > 0:
            adj = O.apply_repetition_controls(lg, w, penalty, ngram)
        want = O.sample(adj, temperature, top_k, uni[i])
        assert got[i] == want, f"row {i}: device {got[i]} oracle {want}"


def test_sampler_reference_known_answers(pkg, O, golden):
    """InferenceTests.cs:19-36 on the device sampler."""
    for key in ("greedy_zero_temperature", "top_k_one_is_argmax"):
        g = golden[key]
        V = len(g["logits"])
        _, _, be = make(pkg, O, (V, 8, 16, 1, 2), 1)
        r = pkg.DotNetRandom(g["seed"])
        with be:
            for _ in range(5):
                assert pkg.Sampler.sample(be, np.array(g["logits"], np.float32), g["temperature"], g["top_k"],
                                          r) == g["expected"]


# ---------------------------------------------------------------------------
def check_ids(O, ocfg, params, prompt, got, want, tie=1e-4):
    """Exact, or diverging only at an oracle near-tie."""
    got, want = list(map(int, got)), list(map(int, want))
    if got == want:
        return
    n = next(i for i in range(min(len(got), len(want))) if got[i] != want[i])
    window = (list(prompt) + want[:n])[-ocfg.context_length:]
    lg = O.forward_last(ocfg, params, window)
    gap = abs(float(lg[got[n]]) - float(lg[want[n]]))
    assert gap <= tie * max(1.0, abs(float(lg[want[n]]))), \
        f"ids diverge at step {n} (device {got[n]}, oracle {want[n]}) with logit gap {gap}"


def test_generate_c1_greedy_with_slide(pkg, O):
    """tiny model, prompt 32, 256 greedy steps; the last
    31 steps re-prefill the sliding window (Sampler.cs:93-94)."""
    ocfg, params, be = make(pkg, O, C1, 1234)
    prompt = np.random.default_rng(42).integers(0, C1[0], 32).astype(np.int32)
    want = O.generate(ocfg, params, prompt, 256, 0.0, 0, O.DotNetRandom(1))
    with be:
        got = be.generate(prompt.tolist(), 256, 0.0, 0, None)
        st = be.stats()
    assert len(got) == 256
    assert st["reprefills"] == 31
    check_ids(O, ocfg, params, prompt, got, want)


def test_generate_sampled_controls(pkg, O):
    """Sampled decode with temperature, top-k, repetition penalty and
    no-repeat-ngram (the Forge-98M bs1 options) on a small model."""
    shape = (2256, 96, 128, 2, 4)
    ocfg, params, be = make(pkg, O, shape, 5)
    prompt = np.random.default_rng(1).integers(0, shape[0], 20).astype(np.int32)
    want = O.generate(ocfg, params, prompt, 120, 0.7, 30, O.DotNetRandom(77), repetition_penalty=1.1,
                      no_repeat_ngram=4)
    r = pkg.DotNetRandom(77)
    with be:
        got = be.generate(prompt.tolist(), 120, 0.7, 30, r, repetition_penalty=1.1, no_repeat_ngram_size=4)
    assert r.draws == len(got)  # one draw per sampled token (Sampler.cs:61)
    check_ids(O, ocfg, params, prompt, got, want)


def test_forge98m_vocabulary_persistent_and_graph_paths(pkg, O, monkeypatch):
    """The Forge-98M vocabulary (V 16384: 148 slices of 111 entries) on a
    small body, through the persistent decode kernel and, with
    FORGE_B200_DECODE=graph, through the CUDA-graph step: teacher-forced
    logits and sampled ids with every repetition control."""
    shape = (16384, 160, 128, 2, 2)
    ocfg = O.Config(*shape)
    params = O.init_params(ocfg, 21)
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, shape[0], 40).astype(np.int32)
    toks = rng.integers(0, shape[0], (1, 72)).astype(np.int32)
    want = O.generate(ocfg, params, prompt, 90, 0.7, 30, O.DotNetRandom(5), repetition_penalty=1.1,
                      no_repeat_ngram=4)
    for mode in ("persistent", "graph"):
        if mode == "graph":
            monkeypatch.setenv("FORGE_B200_DECODE", "graph")
        be = pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0])
        with be:
            got = be.generate(prompt.tolist(), 90, 0.7, 30, pkg.DotNetRandom(5), repetition_penalty=1.1,
                              no_repeat_ngram_size=4)
            tf = be.teacher_forced_logits(toks, 40)
        check_ids(O, ocfg, params, prompt, got, want)
        for k in (0, 13, 31):
            assert relerr(tf[0, k], O.forward_last(ocfg, params, toks[0, :40 + k])) <= TOL, (mode, k)


def test_full_context_prompts_reprefill_every_step(pkg, O):
    """The forge-220m bs16 pattern on a small model:
    prompts fill the context, so every sampled token slides the window and
    re-forwards it (Sampler.cs:93-94) -- the tensor-core GEMM and the
    register-tiled attention prefill on every step."""
    shape = (600, 64, 64, 2, 2)
    ocfg = O.Config(*shape)
    params = O.init_params(ocfg, 31)
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, shape[0], 64).astype(np.int32) for _ in range(3)]
    seeds = [7, 8, 9]
    be = pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0], max_seqs=3)
    with be:
        got = be.generate_batch([p.tolist() for p in prompts], 20, 0.7, 30, seeds=seeds)
        st = be.stats()
    assert st["reprefills"] == 3 * 19
    for i, p in enumerate(prompts):
        want = O.generate(ocfg, params, p, 20, 0.7, 30, O.DotNetRandom(seeds[i]))
        check_ids(O, ocfg, params, p, got[i], want)


def test_bf16_weights(pkg, O, monkeypatch):
    """FB2_WEIGHTS_BF16 (the Forge-98M bf16 config): the
    library computes with tok_emb and the projections rounded to bf16.  Against
    the oracle run on the same rounded weights the fp32 bar holds (logits
    1e-3, ids exact or near-tie) on every path -- persistent kernel and graph
    step, the bf16 gemv and head, prefill; against the fp32 model the stated
    C5 tolerance is logits max-rel <= 2e-2."""
    shape = (16384, 160, 128, 2, 2)
    ocfg = O.Config(*shape)
    params = O.init_params(ocfg, 41)
    rparams = O.round_bf16(ocfg, params)
    rng = np.random.default_rng(17)
    toks = rng.integers(0, shape[0], (2, 60)).astype(np.int32)
    prompts = [rng.integers(0, shape[0], L).astype(np.int32) for L in (20, 33, 47)]
    batch20 = [rng.integers(0, shape[0], 5 + i).astype(np.int32) for i in range(20)]
    for mode in ("persistent", "graph"):
        if mode == "graph":
            monkeypatch.setenv("FORGE_B200_DECODE", "graph")
        be = pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0], max_seqs=20, weight_dtype="bf16")
        with be:
            tf = be.teacher_forced_logits(toks, 40)
            got1 = be.generate(prompts[0].tolist(), 40, 0.7, 30, pkg.DotNetRandom(3), repetition_penalty=1.1,
                               no_repeat_ngram_size=4)
            gotb = be.generate_batch([p.tolist() for p in prompts], 24, 0.0, 0)
            got20 = be.generate_batch([p.tolist() for p in batch20], 6, 0.0, 0)  # decode rows on the tensor cores
        for s_ in range(2):
            for k in (0, 9, 20):
                want = O.forward_last(ocfg, rparams, toks[s_, :40 + k])
                assert relerr(tf[s_, k], want) <= TOL, (mode, s_, k)
                full = O.forward_last(ocfg, params, toks[s_, :40 + k])
                assert relerr(tf[s_, k], full) <= 2e-2, (mode, s_, k)
        want1 = O.generate(ocfg, rparams, prompts[0], 40, 0.7, 30, O.DotNetRandom(3), repetition_penalty=1.1,
                           no_repeat_ngram=4)
        check_ids(O, ocfg, rparams, prompts[0], got1, want1)
        for i, p in enumerate(prompts):
            check_ids(O, ocfg, rparams, p, gotb[i], O.generate(ocfg, rparams, p, 24, 0.0, 0, O.DotNetRandom(1)))
        if mode == "graph":
            for i, p in enumerate(batch20):
                check_ids(O, ocfg, rparams, p, got20[i], O.generate(ocfg, rparams, p, 6, 0.0, 0, O.DotNetRandom(1)))


def test_forgemodel_checkpoint_round_trip(pkg, O, tmp_path):
    """CheckpointTests.cs:31-60 on the device: a model loaded from its
    FORGEMODEL1 file gives bitwise the logits of the in-memory model."""
    shape = (300, 24, 32, 2, 2)
    cfg = pkg.ModelConfig(*shape)
    params = O.init_params(O.Config(*shape), 42)
    path = tmp_path / "forge-test.forgemodel"
    pkg.write_forgemodel(path, cfg, params, "Forge-Test")
    toks = np.random.default_rng(2).integers(0, shape[0], (2, 20)).astype(np.int32)
    with pkg.B200Backend(cfg, params, devices=[0], max_seqs=2) as a:
        want = a.forward_last_batch([t.tolist() for t in toks])
    with pkg.B200Backend.from_forgemodel(path, devices=[0], max_seqs=2) as b:
        assert b.config.d_model == shape[2]
        got = b.forward_last_batch([t.tolist() for t in toks])
    assert np.array_equal(np.asarray(got).view(np.uint32), np.asarray(want).view(np.uint32))


def test_chat_turns_reuse_the_cached_prefix(pkg, O):
    """Chat (Program.cs:736-765) resubmits the whole history each turn: the
    second turn prefills only the positions the first turn did not leave in
    the cache, and its ids are those of a fresh generate.  A prompt that
    departs from the history reuses only the common prefix."""
    shape = (2256, 96, 128, 2, 4)
    ocfg, params, be = make(pkg, O, shape, 5)
    rng = np.random.default_rng(4)
    p1 = rng.integers(0, shape[0], 20).astype(np.int32).tolist()
    with be:
        g1 = be.generate(p1, 12, 0.0, 0, None)
        u2 = rng.integers(0, shape[0], 7).astype(np.int32).tolist()
        p2 = p1 + list(g1) + u2
        be.reset_stats()
        g2 = be.generate(p2, 12, 0.0, 0, None)
        st = be.stats()
        assert st["reused_prefix_rows"] == len(p1) + len(g1) - 1
        assert st["prefill_rows"] == len(p2) - st["reused_prefix_rows"]
        check_ids(O, ocfg, params, np.array(p2), g2, O.generate(ocfg, params, np.array(p2), 12, 0.0, 0,
                                                                 O.DotNetRandom(1)))
        p3 = p2[:10] + [(p2[10] + 1) % shape[0]] + p2[11:]  # an edit at position 10
        be.reset_stats()
        g3 = be.generate(p3, 8, 0.7, 30, pkg.DotNetRandom(9))
        assert be.stats()["reused_prefix_rows"] == 10
        check_ids(O, ocfg, params, np.array(p3), g3, O.generate(ocfg, params, np.array(p3), 8, 0.7, 30,
                                                                 O.DotNetRandom(9)))


def test_in_process_sharding_over_two_devices(pkg, O):
    """One model on two GPUs (fb2_model_create with a devices list): the
    sequences of a batch split over the devices' sessions, one host thread
    per device, no collective; ids and logits as on one device."""
    if pkg.device_count() < 2:
        pytest.skip("needs two GPUs")
    shape = (2256, 96, 128, 2, 4)
    ocfg = O.Config(*shape)
    params = O.init_params(ocfg, 5)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, shape[0], L).astype(np.int32) for L in (9, 30, 17, 44, 5)]
    seeds = [11, 12, 13, 14, 15]
    with pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0, 1], max_seqs=5) as be:
        assert be.stats()["device_count"] == 2
        got = be.generate_batch([p.tolist() for p in prompts], 16, 0.7, 30, seeds=seeds, repetition_penalty=1.1,
                                no_repeat_ngram_size=3)
        lg = be.forward_last_batch([p.tolist() for p in prompts])
    for i, p in enumerate(prompts):
        want = O.generate(ocfg, params, p, 16, 0.7, 30, O.DotNetRandom(seeds[i]), repetition_penalty=1.1,
                          no_repeat_ngram=3)
        check_ids(O, ocfg, params, p, got[i], want)
        assert relerr(lg[i], O.forward_last(ocfg, params, p)) <= TOL


def test_batched_head_and_decode_24_sequences(pkg, O):
    """More than 16 rows reach the head: the tied head runs as one
    tensor-core pass over tok_emb (prefill slots and decode batch), the
    projections as the swapped-operand GEMM."""
    shape = (2256, 64, 128, 2, 4)
    ocfg, params, be = make(pkg, O, shape, 8, max_seqs=24)
    rng = np.random.default_rng(31)
    prompts = [rng.integers(0, shape[0], int(rng.integers(1, 50))).astype(np.int32) for _ in range(24)]
    with be:
        lg = be.forward_last_batch([p.tolist() for p in prompts])
        got = be.generate_batch([p.tolist() for p in prompts], 10, 0.0, 0)
    for i, p in enumerate(prompts):
        assert relerr(lg[i], O.forward_last(ocfg, params, p)) <= TOL, i
        check_ids(O, ocfg, params, p, got[i], O.generate(ocfg, params, p, 10, 0.0, 0, O.DotNetRandom(1)))


def test_generate_batch_ragged_and_long_prompts(pkg, O):
    shape = (300, 24, 32, 2, 2)
    ocfg, params, be = make(pkg, O, shape, 9, max_seqs=5)
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 300, L).astype(np.int32) for L in (1, 5, 23, 24, 40)]
    seeds = [3, 4, 5, 6, 7]
    with be:
        got = be.generate_batch([p.tolist() for p in prompts], 30, 0.9, 20, seeds=seeds, repetition_penalty=1.2,
                                no_repeat_ngram_size=2)
    for i, p in enumerate(prompts):
        want = O.generate(ocfg, params, p, 30, 0.9, 20, O.DotNetRandom(seeds[i]), repetition_penalty=1.2,
                          no_repeat_ngram=2)
        check_ids(O, ocfg, params, p, got[i], want)


def test_generate_reference_behaviours(pkg, O, golden):
    """InferenceTests.cs:80-112, 145-172 on the device path."""
    g = golden["generate_count_in_range"]
    ocfg, params, be = make(pkg, O, tuple(g["config"]), g["model_seed"])
    with be:
        out = be.generate(g["prompt"], g["max_new"], g["temperature"], g["top_k"], pkg.DotNetRandom(g["rng_seed"]))
        assert len(out) == g["max_new"] and all(0 <= t < 32 for t in out)
        want = O.generate(ocfg, params, g["prompt"], g["max_new"], 1.0, 0, O.DotNetRandom(g["rng_seed"]))
        check_ids(O, ocfg, params, g["prompt"], out, want)
        with pytest.raises(ValueError):
            be.generate([1], 1, 1.0, 0, pkg.DotNetRandom(1), repetition_penalty=0.9)
        with pytest.raises(ValueError):
            be.generate([1], -1, 1.0, 0, pkg.DotNetRandom(1))
        with pytest.raises(ValueError):
            be.generate([], 1, 1.0, 0, pkg.DotNetRandom(1))
        with pytest.raises(ValueError):
            be.generate([32], 1, 0.0, 0, None)
        with pytest.raises(ValueError):
            be.generate([1], 1, 0.0, 0, None, eos_id=32)
    g = golden["generate_slides_window"]
    ocfg, params, be = make(pkg, O, tuple(g["config"]), g["model_seed"])
    prompt = [i % 32 for i in range(g["prompt_len"])]
    with be:
        out = be.generate(prompt, g["max_new"], 0.0, 0, None)
    assert len(out) == g["max_new"]
    check_ids(O, ocfg, params, prompt, out, O.generate(ocfg, params, prompt, g["max_new"], 0.0, 0, O.DotNetRandom(1)))
    g = golden["generate_stops_at_eos"]
    ocfg, params, be = make(pkg, O, tuple(g["config"]), g["model_seed"])
    with be:
        first = be.generate(g["prompt"], 1, 0.0, 0, None)[0]
        out = be.generate(g["prompt"], g["max_new"], 0.0, 0, None, eos_id=first)
    assert out == [first]


def test_streaming_callback_and_session_rng(pkg, O):
    """Per-token callback in step order, early stop, and the session RNG
    carried across calls (chat keeps one Random, Program.cs:730)."""
    shape = (64, 32, 16, 1, 2)
    ocfg, params, be = make(pkg, O, shape, 4)
    seen = []
    with be:
        out = be.generate_batch([[1, 2, 3]], 10, 0.8, 0, seeds=[5],
                                on_token=lambda s, st, t: (seen.append((s, st, t)), st == 6)[1])
        assert [t for _, _, t in seen] == out[0].tolist() and len(out[0]) == 7
        assert [st for _, st, _ in seen] == list(range(7))
    r = O.DotNetRandom(5)
    want = O.generate(ocfg, params, [1, 2, 3], 7, 0.8, 0, r)
    check_ids(O, ocfg, params, [1, 2, 3], out[0], want)


def test_tensor_core_attention_blocks_and_offsets(pkg, O, monkeypatch):
    """The tcgen05 prefill attention (head_dim 64): windows that end on and
    around its 64-key tiles and 128-query blocks, against the oracle and
    against the SIMT kernel (FORGE_B200_ATTN=simt) on the same inputs; and a
    chat turn whose prefill starts inside a query block."""
    shape = (512, 400, 128, 2, 2)  # head_dim 64
    lens = [1, 63, 64, 65, 127, 128, 129, 200, 257, 400]
    rng = np.random.default_rng(17)
    wins = [rng.integers(0, shape[0], L).astype(np.int32) for L in lens]
    ocfg, params, be = make(pkg, O, shape, 3, max_seqs=len(lens))
    with be:
        tc = be.forward_last_batch(wins)
    for i, w in enumerate(wins):
        assert relerr(tc[i], O.forward_last(ocfg, params, w)) <= TOL, f"window len {lens[i]}"
    monkeypatch.setenv("FORGE_B200_ATTN", "simt")
    be2 = pkg.B200Backend(pkg.ModelConfig(*shape), params, devices=[0], max_seqs=len(lens))
    with be2:
        simt = be2.forward_last_batch(wins)
    monkeypatch.delenv("FORGE_B200_ATTN")
    for i in range(len(lens)):
        assert relerr(tc[i], simt[i]) <= 1e-4, f"tensor-core vs SIMT attention, window len {lens[i]}"
    # second chat turn: the cache holds 158 positions, the prefill starts at 157
    ocfg, params, be = make(pkg, O, shape, 4)
    p1 = rng.integers(0, shape[0], 150).astype(np.int32).tolist()
    with be:
        g1 = be.generate(p1, 8, 0.0, 0, None)
        p2 = p1 + list(g1) + rng.integers(0, shape[0], 5).astype(np.int32).tolist()
        be.reset_stats()
        g2 = be.generate(p2, 10, 0.0, 0, None)
        assert be.stats()["reused_prefix_rows"] == len(p1) + len(g1) - 1
    check_ids(O, ocfg, params, np.array(p2), g2, O.generate(ocfg, params, np.array(p2), 10, 0.0, 0, O.DotNetRandom(1)))
