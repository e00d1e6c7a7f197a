"""Pins the CPU oracle against the reference's own known-answer tests
(tests/golden/known_answers.json, each entry citing its source test)."""
from __future__ import annotations

import math

import numpy as np
import pytest


def _f(v):
    return -math.inf if v == "-inf" else float(v)


def test_greedy_and_top_k_one(O, golden):
    for key in ("greedy_zero_temperature", "top_k_one_is_argmax"):
        g = golden[key]
        rng = O.DotNetRandom(g["seed"])
        for _ in range(g["draws"]):
            u = rng.next_double()
            assert O.sample(g["logits"], g["temperature"], g["top_k"], u) == g["expected"], key
    assert O.greedy(np.array(golden["greedy_zero_temperature"]["logits"], np.float32)) == 1


def test_dominant_and_distribution(O, golden):
    g = golden["dominant_logit"]
    rng = O.DotNetRandom(g["seed"])
    hits = sum(O.sample(g["logits"], 1.0, 0, rng.next_double()) == 0 for _ in range(g["draws"]))
    assert hits > g["min_hit_fraction"] * g["draws"]
    g = golden["distribution_matches_softmax"]
    rng = O.DotNetRandom(g["seed"])
    counts = np.zeros(3)
    for _ in range(g["draws"]):
        counts[O.sample(g["logits"], 1.0, 0, rng.next_double())] += 1
    e = np.exp(np.array(g["logits"], np.float32))
    e /= e.sum()
    assert np.all(np.abs(counts / g["draws"] - e) <= g["tolerance"])


def test_top_k_zero_and_above_vocab(O, golden):
    g = golden["top_k_zero_and_above_vocab"]
    rng = O.DotNetRandom(g["seed"])
    for _ in range(g["draws"]):
        for k in g["top_ks"]:
            assert 0 <= O.sample(g["logits"], 1.0, k, rng.next_double()) < 4


@pytest.mark.parametrize("key", ["repetition_penalty", "no_repeat_ngram", "no_repeat_ngram_all_banned_restores"])
def test_repetition_controls(O, golden, key):
    g = golden[key]
    out = O.apply_repetition_controls(g["logits"], g["history"], g["penalty"], g["ngram"])
    exp = np.array([_f(v) for v in g["expected"]], np.float32)
    assert np.array_equal(out, exp), (out, exp)


def test_invalid_options(O):
    with pytest.raises(ValueError):
        O.sample(np.zeros(0, np.float32), 1.0, 0, 0.5)
    with pytest.raises(ValueError):
        O.sample([1.0], float("nan"), 0, 0.5)
    with pytest.raises(ValueError):
        O.apply_repetition_controls([1.0, 2.0], [0], 0.9, 0)
    with pytest.raises(ValueError):
        O.apply_repetition_controls([1.0, 2.0], [0], 1.0, -1)
    cfg = O.Config(32, 8, 16, 2, 2)
    p = O.init_params(cfg, 2)
    with pytest.raises(ValueError):
        O.generate(cfg, p, [1], 1, 1.0, 0, O.DotNetRandom(1), repetition_penalty=0.9)
    with pytest.raises(ValueError):
        O.generate(cfg, p, [1], -1, 1.0, 0, O.DotNetRandom(1))
    with pytest.raises(ValueError):
        O.forward_last(cfg, p, [32])  # token out of range (GptModel.cs:288-299)


def test_gelu_softmax_layernorm(O, golden):
    g = golden["gelu_known_values"]
    y = O.gelu(g["x"])
    assert np.max(np.abs(y - np.array(g["expected"], np.float32))) <= g["tolerance"]
    g = golden["softmax_rows_sum_to_one"]
    rng = O.DotNetRandom(g["seed"])
    x = np.array([rng.next_double() * 20 - 10 for _ in range(g["rows"] * g["cols"])], np.float32)
    raw = x.copy()
    x[0] = g["extreme"]
    y = O.softmax_rows(x.reshape(g["rows"], g["cols"]))
    assert np.all(np.abs(y.sum(1) - 1) <= g["tolerance"])
    e = np.exp(raw[2 * g["cols"]:].astype(np.float64))
    assert np.max(np.abs(y[2] - e / e.sum())) <= g["tolerance"]
    assert y[0, 0] > 0.99
    g = golden["layer_norm_normalizes_rows"]
    r = np.random.default_rng(7)
    x = (r.standard_normal((g["rows"], g["cols"])) * 3).astype(np.float32)
    y = O.layer_norm(x, np.ones(g["cols"], np.float32), np.zeros(g["cols"], np.float32))
    assert np.all(np.abs(y.mean(1)) <= g["mean_tolerance"])
    assert np.all(np.abs(y.var(1) - 1) <= g["var_tolerance"])


def test_model_shapes_and_forward_last(O, golden):
    g = golden["small_model_param_count"]
    cfg = O.Config(*g["config"])
    p = O.init_params(cfg, 1)
    assert sum(a.size for a in p) == g["expected"]
    assert not any(n.startswith("head.") for n in O.param_names(cfg))
    full = O.forward(cfg, p, g["tokens"])
    last = O.forward_last(cfg, p, g["tokens"])
    assert full.shape == (len(g["tokens"]), cfg.vocab_size)
    assert np.array_equal(full[-1], last)  # exact (ModelTests.cs:37-39)


def test_forward_deterministic_per_seed(O, golden):
    g = golden["forward_deterministic_per_seed"]
    cfg = O.Config(*g["config"])
    a, b, c = (O.forward(cfg, O.init_params(cfg, s), g["tokens"]) for s in g["seeds"])
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)


def test_init_residual_std(O, golden):
    g = golden["init_residual_std"]
    cfg = O.Config(*g["config"])
    p = dict(zip(O.param_names(cfg), O.init_params(cfg, g["seed"])))
    proj_std = np.float32(0.02) / np.sqrt(np.float32(2 * cfg.n_layers))
    for name in g["tensors"]:
        w = p[name].astype(np.float64)
        exp = proj_std if "proj" in name else g["std"]
        assert g["band"][0] * exp < w.std() < g["band"][1] * exp, name
    assert np.all(p["blocks.0.ln1.w"] == 1) and np.all(p["ln_f.b"] == 0)


def test_generate_count_slide_eos(O, golden):
    g = golden["generate_count_in_range"]
    cfg = O.Config(*g["config"])
    p = O.init_params(cfg, g["model_seed"])
    out = O.generate(cfg, p, g["prompt"], g["max_new"], g["temperature"], g["top_k"], O.DotNetRandom(g["rng_seed"]))
    assert len(out) == g["max_new"] and np.all((out >= 0) & (out < cfg.vocab_size))
    g = golden["generate_slides_window"]
    p = O.init_params(cfg, g["model_seed"])
    prompt = [i % cfg.vocab_size for i in range(g["prompt_len"])]
    out = O.generate(cfg, p, prompt, g["max_new"], 0.0, 0, O.DotNetRandom(g["rng_seed"]))
    assert len(out) == g["max_new"]
    g = golden["generate_stops_at_eos"]
    p = O.init_params(cfg, g["model_seed"])
    first = O.generate(cfg, p, g["prompt"], 1, 0.0, 0, O.DotNetRandom(g["rng_seed"]))[0]
    out = O.generate(cfg, p, g["prompt"], g["max_new"], 0.0, 0, O.DotNetRandom(g["rng_seed"]), eos_id=int(first))
    assert list(out) == [first]


def test_generate_equals_stepwise_forward(O):
    """The loop restatement: each step samples from ForwardLast of the
    truncated window (Sampler.cs:91-108), drawing one uniform per token."""
    cfg = O.Config(40, 10, 16, 2, 2)
    p = O.init_params(cfg, 3)
    prompt = [1, 7, 3]
    ids, logits = O.generate(cfg, p, prompt, 12, 0.8, 5, O.DotNetRandom(9), repetition_penalty=1.3,
                             no_repeat_ngram=2, return_logits=True)
    rng = O.DotNetRandom(9)
    window = list(prompt)
    for n, tok in enumerate(ids):
        window = window[-cfg.context_length:]
        lg = O.forward_last(cfg, p, window)
        assert np.array_equal(lg, logits[n])
        assert O.sample_step(lg, window, 0.8, 5, 1.3, 2, rng) == tok
        window.append(int(tok))


def test_dotnet_random_restatements_agree(O, pkg):
    """Oracle C, package Python and library C++ restatements of
    `new Random(seed)` produce the same stream (the .NET stream itself is
    not pinned: no .NET runtime here)."""
    import ctypes as C
    from forge_lm_b200 import _native as N
    for seed in (0, 1, 42, 1234, -7, 2**31 - 1, -2**31):
        a = O.DotNetRandom(seed).next_doubles(200)
        r = pkg.DotNetRandom(seed)
        b = np.array([r.next_double() for _ in range(200)])
        c = np.empty(200, np.float64)
        N.check(N.load().fb2_test_dotnet_random(seed, 200, C.c_void_p(c.ctypes.data)))
        assert np.array_equal(a, b) and np.array_equal(a, c), seed
        assert np.all((a >= 0) & (a < 1))


def test_round_bf16_ties_to_even_and_scope(O):
    """round_bf16: nearest-even bf16 of the projections and tok_emb only."""
    cfg = O.Config(12, 6, 8, 1, 2)
    params = O.init_params(cfg, 3)
    r = O.round_bf16(cfg, params)
    bits = [np.float32(1.0 + 2.0 ** -8), np.float32(1.0 + 3 * 2.0 ** -8), np.float32(-2.5 + 2.0 ** -9)]
    want = [np.float32(1.0), np.float32(1.0 + 2 * 2.0 ** -7), np.float32(-2.5)]
    p = [np.array(b, np.float32).reshape(1) for b in bits]
    for b, w in zip(p, want):
        q = O.round_bf16(O.Config(1, 1, 4, 1, 1), [b] + [np.zeros(1, np.float32)] * 15)[0]
        assert q[0] == w
    for i, (a, b) in enumerate(zip(params, r)):
        narrowed = i == 0 or (i >= 2 and (i - 2) % 12 in (2, 4, 8, 10) and i < 2 + 12 * cfg.n_layers)
        if narrowed:
            assert np.all((b.view(np.uint32) & 0xFFFF) == 0) and np.max(np.abs(a - b)) <= np.max(np.abs(a)) * 2 ** -8
        else:
            assert np.array_equal(a, b)
