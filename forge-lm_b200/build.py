"""Builds libforge_b200.so in-tree for sm_100a (B200).

Steps:
  1. gen_expf_fixups (host gcc) -> csrc/generated/expf_fixups.inc: the inputs
     where the host libm expf differs from the correctly rounded exponential
     (the on-device sampler reproduces the host expf bit for bit).
  2. nvcc -gencode arch=compute_100a,code=sm_100a -> libforge_b200.so.
No fast-math: the sampler's division and exponentials must round as IEEE.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
GEN = os.path.join(CSRC, "generated")
LIB = os.path.join(HERE, "libforge_b200.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def gen_fixups(verbose: bool = False) -> str:
    os.makedirs(GEN, exist_ok=True)
    src = os.path.join(CSRC, "gen_expf_fixups.c")
    out = os.path.join(GEN, "expf_fixups.inc")
    if not _newer(out, [src]):
        return out
    exe = os.path.join(GEN, "gen_expf_fixups")
    subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", src, "-o", exe, "-lm"], check=True)
    r = subprocess.run([exe, out], check=True, capture_output=True, text=True)
    if verbose:
        print(r.stdout.strip())
    os.remove(exe)
    return out


def _flags() -> list[str]:
    """nvcc flags; FORGE_B200_PHASE_TRACE=1 adds the persistent kernel's
    per-phase stamps (a diagnostic build: the stamps cost throughput)."""
    flags = list(NVCC_FLAGS)
    if os.environ.get("FORGE_B200_PHASE_TRACE") == "1":
        flags.append("-DFB2_MK_PHASE_TRACE")
    return flags


def _sources() -> list[str]:
    sources = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".hpp"))]
    sources.append(os.path.join(ROOT, "include", "forge_b200.h"))
    sources.append(os.path.join(GEN, "expf_fixups.inc"))
    return sorted(sources)


def source_fingerprint(flags: list[str], sources: list[str]) -> str:
    """SHA-256 of the nvcc flags and every source file (path and contents):
    names the build independently of the binary, which nvcc does not
    reproduce byte for byte."""
    h = hashlib.sha256(" ".join(flags).encode())
    for path in sources:
        h.update(os.path.relpath(path, ROOT).encode())
        with open(path, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def stamp_path(lib: str = LIB) -> str:
    """The JSON beside the library: the flags and source fingerprint it was built from."""
    return lib + ".flags"


def read_stamp(lib: str = LIB) -> dict:
    try:
        with open(stamp_path(lib)) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def build(verbose: bool = False, force: bool = False) -> str:
    gen_fixups(verbose)
    sources = _sources()
    flags = _flags()
    same_flags = read_stamp().get("flags") == flags
    if not force and same_flags and not _newer(LIB, sources):
        return LIB
    cmd = [_nvcc(), *flags, "-shared", "-o", LIB + ".tmp", os.path.join(CSRC, "forge_b200.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    with open(stamp_path(), "w") as f:
        json.dump({"flags": flags, "sources_sha256": source_fingerprint(flags, sources)}, f)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
