"""The algorithmic bytes and FLOPs behind bench.py's roofline figures, checked
against the model definition rather than against themselves: the weights a
decode step streams are every parameter except pos_emb (one row of it per
sequence goes with the sequence's bytes), and one sliding-window step is the
block projections for every row, causal attention over T(T+1)/2 pairs, and
the head on the last row."""
import os

import numpy as np

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_weight_bytes_are_the_parameters_a_step_streams(pkg):
    for m in (bench.FORGE_98M, bench.FORGE_220M):
        cfg = pkg.ModelConfig(m["vocab_size"], m["context_length"], m["d_model"], m["n_layers"], m["n_heads"])
        sizes = {n: int(np.prod(s)) for n, s in zip(pkg.param_names(cfg), pkg.param_shapes(cfg))}
        streamed = sum(v for n, v in sizes.items() if n != "pos_emb")
        assert bench.weight_bytes(m) == 4.0 * streamed
        # bf16: the projections and the tied head narrow to 2 bytes, the
        # biases and LayerNorm parameters stay fp32
        wide = sum(v for n, v in sizes.items() if n == "tok_emb" or n.endswith(".w") and "ln" not in n)
        assert bench.weight_bytes(m, "bf16") == 2.0 * wide + 4.0 * (streamed - wide)
    assert abs(bench.weight_bytes(bench.FORGE_98M) / 1e6 - 390.56) < 0.01  # the figure the docs quote


def test_sequence_bytes_and_window_flops():
    m = bench.FORGE_98M
    D, L, V, F = m["d_model"], m["n_layers"], m["vocab_size"], 4 * m["d_model"]
    for T in (1, 64, 576, 1024):
        # token + position rows, and K and V of T positions in every layer
        assert bench.sequence_bytes(m, T) == 4.0 * (2 * D + 2 * L * T * D)
        per_row = 2 * (D * 3 * D + D * D + D * F + F * D)  # qkv, proj, fc, mlp proj
        pairs = T * (T + 1) // 2
        attn = L * 2 * (2 * pairs * D)  # scores and context, 2 FLOPs per multiply-add
        assert bench.flops_per_sequence_step(m, T) == T * L * per_row + attn + 2 * D * V


def test_reference_step_flops_and_cpu_sample_on_a_tiny_workload(O):
    """The reference step's cost model counts every row through the blocks,
    the full T x T scores and context, and every row's logits; the CPU leg
    returns its ids (for the bench's parity field) and a full-run estimate."""
    m = dict(vocab_size=300, context_length=32, d_model=32, n_layers=2, n_heads=2)
    D, L, V = 32, 2, 300
    assert bench.ref_flops_per_token(m, 10) == 2.0 * 10 * (L * 12 * D * D + V * D) + 4.0 * L * 100 * D
    wl = dict(name="tiny", model=m, prompt_len=8, new_tokens=40, temperature=0.7, top_k=5, penalty=1.1, ngram=2)
    r = bench.cpu_reference_sample(wl, n_tokens=6)
    assert len(r["ids"]) == 6 and r["value"] > 0 and r["cpu_model"]
    assert r["full_run"]["value"] > 0
    want = O.generate(O.Config(300, 32, 32, 2, 2), O.init_params(O.Config(300, 32, 32, 2, 2), bench.WEIGHT_SEED),
                      bench.prompts_for(0, 1, 8, 300)[0], 6, 0.7, 5, O.DotNetRandom(1), repetition_penalty=1.1,
                      no_repeat_ngram=2)
    assert list(r["ids"]) == list(want)
    p = bench.parity_vs_cpu(list(want) + [7, 7], r["ids"])
    assert p["ids_equal"] == 6 and p["first_mismatch"] is None
    p = bench.parity_vs_cpu([int(want[0]) + 1] + list(want[1:]), r["ids"])
    assert p["first_mismatch"] == 0 and p["ids_equal"] == 5


def test_traffic_record_is_keyed_by_the_build(tmp_path, monkeypatch):
    """A DRAM-traffic figure is reported only for a library built from the
    sources and flags it was measured on (the build's fingerprint, written
    beside the library)."""
    lib = tmp_path / "lib.so"
    lib.write_bytes(b"binary")
    stamp = tmp_path / "lib.so.flags"
    stamp.write_text('{"flags": [], "sources_sha256": "aaa"}')
    rec = tmp_path / "traffic.json"
    monkeypatch.setattr(bench, "TRAFFIC_RECORD", str(rec))
    rec.write_text('{"c2": {"dram_bytes_per_step": 123.0, "build_sha256": "aaa"}}')
    assert bench.recorded_traffic("c2", str(lib)) == 123.0
    assert bench.recorded_traffic("c3", str(lib)) is None
    stamp.write_text('{"flags": [], "sources_sha256": "bbb"}')
    assert bench.recorded_traffic("c2", str(lib)) is None
    stamp.unlink()
    assert bench.recorded_traffic("c2", str(lib)) is None


def test_build_fingerprint_follows_sources_and_flags(tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("fb2_build", os.path.join(ROOT, "forge-lm_b200", "build.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    src = tmp_path / "k.cu"
    src.write_text("int x;")
    f1 = b.source_fingerprint(["-O3"], [str(src)])
    assert f1 == b.source_fingerprint(["-O3"], [str(src)])
    assert f1 != b.source_fingerprint(["-O2"], [str(src)])
    src.write_text("int y;")
    assert f1 != b.source_fingerprint(["-O3"], [str(src)])


def test_reference_arm_prints_the_same_config(monkeypatch, capsys):
    """Both arms' lines carry the same `config` object (the driver compares
    them), whatever the rank count."""
    import json
    import types
    fake = {"value": 1.0, "unit": "tokens/s", "cores": 1, "cpu_model": "x", "kind": "port", "sample": "s",
            "seconds": 1.0, "ids": [1, 2]}
    monkeypatch.setattr(bench, "cpu_reference_sample", lambda wl, full_run=True: dict(fake))
    for world in (1, 2):
        monkeypatch.setattr(bench, "dist_env", lambda w=world: (0, w, 0))
        wl = dict(bench.WORKLOADS["c3"])
        bench.run_reference(types.SimpleNamespace(warmup=1, steps=1), wl)
        line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert line["impl"] == "reference"
        assert line["config"] == bench.workload_config(wl, world)
    assert bench.workload_config(dict(bench.WORKLOADS["c3"]), 2)["sequences_per_gpu"] == 32
