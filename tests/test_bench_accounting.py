"""The algorithmic bytes and FLOPs behind bench.py's roofline figures, checked
against the model definition rather than against themselves: the weights a
decode step streams are every parameter except pos_emb (one row of it per
sequence goes with the sequence's bytes), and one sliding-window step is the
block projections for every row, causal attention over T(T+1)/2 pairs, and
the head on the last row."""
import numpy as np

import bench


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
