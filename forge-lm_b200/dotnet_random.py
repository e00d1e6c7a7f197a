"""The uniform stream of `new System.Random(seed)` for the Python host mirror.

The reference sampler draws one (float)rng.NextDouble() per sampled token
(src/LLM.Core/Inference/Sampler.cs:61).  .NET seeds `new Random(seed)` with
the published subtractive generator of Knuth (TAOCP vol. 2, 3.2.2) in its
"compat" variant; NextDouble() = sample * (1.0 / int.MaxValue).  The same
restatement lives in the C++ library (csrc/dotnet_random.hpp) for the
FB2_RNG_SEEDS / FB2_RNG_SESSION modes.  No .NET runtime exists on this build
host, so agreement with a real .NET stream is not pinned by a test here.
"""
from __future__ import annotations

_BIG = 2147483647
_SEED = 161803398


def _wrap(x: int) -> int:
    """C# int arithmetic wraps (unchecked context)."""
    return ((x + 2**31) & 0xFFFFFFFF) - 2**31


class DotNetRandom:
    __slots__ = ("_t", "_a", "_b", "draws")

    def __init__(self, seed: int = 0):
        seed = int(seed)
        if not -2**31 <= seed < 2**31:
            raise ValueError("seed must be an int32")
        t = [0] * 56
        sub = _BIG if seed == -2**31 else abs(seed)
        mj = _SEED - sub
        t[55] = mj
        mk, ii = 1, 0
        for _ in range(1, 55):
            ii += 21
            if ii >= 55:
                ii -= 55
            t[ii] = mk
            mk = _wrap(mj - mk)
            if mk < 0:
                mk = _wrap(mk + _BIG)
            mj = t[ii]
        for _ in range(1, 5):
            for i in range(1, 56):
                n = i + 30
                if n >= 55:
                    n -= 55
                t[i] = _wrap(t[i] - t[1 + n])
                if t[i] < 0:
                    t[i] = _wrap(t[i] + _BIG)
        self._t, self._a, self._b, self.draws = t, 0, 21, 0

    def clone(self) -> "DotNetRandom":
        c = DotNetRandom.__new__(DotNetRandom)
        c._t, c._a, c._b, c.draws = list(self._t), self._a, self._b, self.draws
        return c

    def next_sample(self) -> int:
        a = self._a + 1
        if a >= 56:
            a = 1
        b = self._b + 1
        if b >= 56:
            b = 1
        v = _wrap(self._t[a] - self._t[b])
        if v == _BIG:
            v -= 1
        if v < 0:
            v = _wrap(v + _BIG)
        self._t[a] = v
        self._a, self._b = a, b
        self.draws += 1
        return v

    def next_double(self) -> float:
        return self.next_sample() * (1.0 / _BIG)
