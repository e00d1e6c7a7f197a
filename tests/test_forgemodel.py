"""FORGEMODEL1 checkpoints through the library (no device needed).

Restates the reference's checkpoint tests (tests/LLM.Core.Tests/
CheckpointTests.cs: bitwise round trip :31-60, bad magic :131-144, truncated
payload :146-165, same-size corruption fails the checksum :202-240) and the
format rules of Checkpoint.LoadCore (src/LLM.Core/Checkpoint/Checkpoint.cs:
174-264), with an independent writer in this file (json + hashlib) as the
cross-check of the library's reader, writer and SHA-256.
"""
import hashlib
import json
import struct

import numpy as np
import pytest

SMALL = (32, 8, 16, 2, 2)  # CheckpointTests.cs:19


@pytest.fixture(scope="module")
def nat(pkg):
    from forge_lm_b200 import _native
    return _native


def sha256_lib(nat, data: bytes) -> bytes:
    out = (np.zeros(32, np.uint8))
    buf = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    nat.check(nat.load().fb2_test_sha256(buf.ctypes.data, len(data), out.ctypes.data))
    return out.tobytes()


def test_sha256_known_answers(nat):
    """FIPS 180-4 examples and long inputs against hashlib."""
    assert sha256_lib(nat, b"abc").hex() == hashlib.sha256(b"abc").hexdigest()
    assert sha256_lib(nat, b"").hex() == hashlib.sha256(b"").hexdigest()
    msg = b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq"
    assert sha256_lib(nat, msg).hex() == hashlib.sha256(msg).hexdigest()
    rng = np.random.default_rng(5)
    for n in (55, 56, 63, 64, 65, 119, 120, 1000, 1 << 20):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert sha256_lib(nat, data) == hashlib.sha256(data).digest(), n


def python_writer(path, cfg, params, name, names=None, architecture="forge-gpt2-tied-v1", training=True):
    """Independent FORGEMODEL1 writer (the layout of Checkpoint.cs:143-166)."""
    header = {"VocabSize": cfg.vocab_size, "ContextLength": cfg.context_length, "DModel": cfg.d_model,
              "NLayers": cfg.n_layers, "NHeads": cfg.n_heads, "ModelName": name, "Architecture": architecture,
              "Names": names if names is not None else param_names_of(cfg)}
    if training:
        header["Training"] = {"GlobalStep": 3, "AdamStep": 0, "HasOptimizerState": False, "MaxLr": 0.001,
                              "DataIdentity": None, "TokenizerIdentity": "tok"}
    js = json.dumps(header, separators=(",", ":")).encode()
    body = b"FORGEMODEL1" + struct.pack("<i", len(js)) + js + b"".join(
        np.ascontiguousarray(p, np.float32).tobytes() for p in params)
    with open(path, "wb") as f:
        f.write(body + hashlib.sha256(body).digest())


def param_names_of(cfg):
    import forge_lm_b200 as m
    return m.param_names(cfg)


def test_round_trip_bitwise_and_layout(pkg, O, tmp_path):
    """CheckpointTests.cs:31-60: config, name and every weight bit round-trip;
    the file layout and trailer are what the reference writes."""
    cfg = pkg.ModelConfig(*SMALL)
    params = O.init_params(O.Config(*SMALL), 42)
    p = tmp_path / "m.forgemodel"
    pkg.write_forgemodel(p, cfg, params, "Forge-Test")
    raw = p.read_bytes()
    assert raw[:11] == b"FORGEMODEL1"
    (jlen,) = struct.unpack("<i", raw[11:15])
    header = json.loads(raw[15:15 + jlen])
    assert (header["VocabSize"], header["ContextLength"], header["DModel"], header["NLayers"], header["NHeads"]) == SMALL
    assert header["ModelName"] == "Forge-Test" and header["Architecture"] == "forge-gpt2-tied-v1"
    assert header["Names"] == pkg.param_names(cfg)
    assert header["Training"]["HasOptimizerState"] is False
    payload = raw[15 + jlen:-32]
    assert payload == b"".join(np.ascontiguousarray(a, np.float32).tobytes() for a in params)
    assert raw[-32:] == hashlib.sha256(raw[:-32]).digest()
    got_cfg, got_name = pkg.read_forgemodel_header(p)
    assert (got_cfg.vocab_size, got_cfg.context_length, got_cfg.d_model, got_cfg.n_layers, got_cfg.n_heads) == SMALL
    assert got_name == "Forge-Test"


def test_reads_an_independently_written_file(pkg, O, tmp_path):
    cfg = pkg.ModelConfig(*SMALL)
    params = O.init_params(O.Config(*SMALL), 7)
    p = tmp_path / "py.forgemodel"
    python_writer(p, cfg, params, "Forge-été \"q\"")
    got_cfg, name = pkg.read_forgemodel_header(p)
    assert name == "Forge-été \"q\"" and got_cfg.d_model == SMALL[2]


@pytest.mark.parametrize("case", ["bad_magic", "truncated", "same_size_corruption", "architecture", "no_training",
                                  "names", "blank_name", "header_length", "json_garbage", "too_short",
                                  "trailing_data"])
def test_rejections_are_invalid_data(pkg, O, tmp_path, case):
    """Each rule of Checkpoint.LoadCore fails loudly as InvalidDataError
    (InvalidDataException in the reference)."""
    cfg = pkg.ModelConfig(*SMALL)
    params = O.init_params(O.Config(*SMALL), 1)
    p = tmp_path / f"{case}.forgemodel"
    pkg.write_forgemodel(p, cfg, params, "Forge-Test")
    raw = bytearray(p.read_bytes())
    if case == "bad_magic":  # CheckpointTests.cs:131-144
        raw = bytearray(b"NOTACHECKPOINT!")
    elif case == "truncated":  # CheckpointTests.cs:146-165
        raw = raw[:-4]
    elif case == "same_size_corruption":  # CheckpointTests.cs:202-240
        raw[len(raw) // 2] ^= 0x40
    elif case == "trailing_data":
        raw += b"\x00" * 4
    elif case == "too_short":
        raw = raw[:20]
    elif case == "header_length":
        raw[11:15] = struct.pack("<i", (1 << 20) + 1)
    elif case == "json_garbage":
        (jlen,) = struct.unpack("<i", raw[11:15])
        raw[15:15 + jlen] = b"{" * jlen
        body = bytes(raw[:-32])
        raw[-32:] = hashlib.sha256(body).digest()
    else:
        kw = {"architecture": dict(architecture="gpt-something"), "no_training": dict(training=False),
              "names": dict(names=list(reversed(pkg.param_names(cfg)))), "blank_name": {}}[case]
        python_writer(p, cfg, params, "   " if case == "blank_name" else "Forge-Test", **kw)
        raw = bytearray(p.read_bytes())
    p.write_bytes(bytes(raw))
    with pytest.raises(pkg.InvalidDataError):
        pkg.read_forgemodel_header(p)


def test_write_rejects_bad_arguments(pkg, O, tmp_path):
    cfg = pkg.ModelConfig(*SMALL)
    params = O.init_params(O.Config(*SMALL), 1)
    with pytest.raises(pkg.ArgumentError):
        pkg.write_forgemodel(tmp_path / "x", cfg, params, "  ")
    with pytest.raises(pkg.ArgumentError):
        pkg.write_forgemodel(tmp_path / "x", cfg, params[:-1], "Forge")
