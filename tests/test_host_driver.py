"""A C host (tests/host_driver/forge_host.c) drives the library through
include/forge_b200.h the way the C# B200Backend shim does: its own random
stream pulled once per sampled token (FB2_RNG_CALLBACK), tokens streamed
through the token callback, the stream carried across chat turns, an early
stop by the consumer, EOS, and the status -> exception mapping of the
reference (ArgumentException, InvalidDataException)."""
from __future__ import annotations

import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "host_driver", "forge_host.c")


@pytest.fixture(scope="module")
def host_exe(pkg, tmp_path_factory):
    lib_dir = os.path.dirname(pkg.library_path())
    exe = str(tmp_path_factory.mktemp("host") / "forge_host")
    subprocess.run(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
                    "-L", lib_dir, "-lforge_b200", f"-Wl,-rpath,{lib_dir}", "-o", exe], check=True)
    return exe


def _lines(out: str) -> dict:
    got: dict = {}
    for d in (json.loads(ln) for ln in out.splitlines() if ln.startswith("{")):
        got.setdefault(d["case"], {}).update(d)  # a case's status line and its tokens line
    return got


def test_host_driver_without_a_device(host_exe, tmp_path):
    bad = tmp_path / "garbage.forgemodel"
    bad.write_bytes(b"FORGEMODEL1 not really")
    r = subprocess.run([host_exe, "nodevice", str(bad)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    got = _lines(r.stdout)
    assert got["version"]["abi"] == 1
    assert got["garbage_checkpoint"]["exception"] == "InvalidDataException"
    assert got["garbage_checkpoint"]["message_len"] > 0
    assert got["null_session_seed"]["exception"] == "ArgumentException"


@pytest.mark.gpu
def test_host_driver_generate_chat_stop_eos_errors(host_exe, O, tmp_path):
    stream = O.DotNetRandom(5).next_doubles(400)
    upath = tmp_path / "uniforms.bin"
    stream.astype("<f8").tofile(upath)
    r = subprocess.run([host_exe, "run", str(upath), str(len(stream))], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    got = _lines(r.stdout)
    for c in ("init_params", "model_create", "session_create", "generate", "chat_turn2", "early_stop", "eos"):
        assert got[c]["status"] == 0, got[c]
    cfg = O.Config(96, 32, 64, 2, 4)
    params = O.init_params(cfg, 11)
    opts = dict(repetition_penalty=1.1, no_repeat_ngram=3)
    prompt = [5, 17, 3, 42, 8]
    pos = 0

    def oracle(p, n, eos=-1):
        nonlocal pos
        ids = O.generate(cfg, params, p, n, 0.8, 10, uniforms=stream[pos:], eos_id=eos, **opts)
        return [int(t) for t in ids]

    g = got["generate"]
    assert g["tokens"] == oracle(prompt, 20) and g["draws"] == 20
    pos += 20
    hist = prompt + g["tokens"] + [7, 9]
    t2 = got["chat_turn2"]
    assert t2["tokens"] == oracle(hist, 6) and t2["draws"] == 6
    pos += 6
    st = got["early_stop"]
    assert st["tokens"] == oracle(prompt, 20)[:4] and st["draws"] == 4
    pos += 4
    e = got["eos"]
    want = oracle(prompt, 20, eos=g["tokens"][2])
    assert e["tokens"] == want and e["draws"] == len(want)
    for c in ("bad_penalty", "token_out_of_range", "eos_out_of_vocab", "no_rng"):
        assert got[c]["exception"] == "ArgumentException" and got[c]["message_len"] > 0, got[c]
