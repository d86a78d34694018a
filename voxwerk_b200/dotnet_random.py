"""System.Random(int) as voxwerk's Sampler uses it (src/Voxwerk/Talker/Sampler.cs:21).

Restated from the published subtractive-generator method (Knuth, TAOCP Vol. 2 3.2.2; Numerical Recipes ``ran3``)
with .NET's modulus 2^31-1 and second tap 21.  Pure Python: importing it loads no native library, so workload
generation and the CPU reference arm of the benchmark can use it without the GPU sampler.
"""

from __future__ import annotations

from typing import Optional

import numpy as np


class DotNetRandom:
    """System.Random(int seed): Knuth's subtractive generator with .NET's parameters.

    ``next_double()`` is Random.NextDouble(), the one draw Sampler.Select takes per sampled row (Sampler.cs:77).
    ``seed=None`` seeds from the OS, like ``new Random()``.
    """

    _MBIG = 2147483647
    _MSEED = 161803398

    @staticmethod
    def _sub(a: int, b: int) -> int:
        """a - b with C# unchecked int32 wrap-around."""
        return ((a - b + 2**31) % 2**32) - 2**31

    def __init__(self, seed: Optional[int] = None):
        if seed is None:
            seed = int.from_bytes(np.random.default_rng().bytes(4), "little", signed=True)
        seed = int(np.int32(np.int64(seed)))   # C# int arithmetic wraps (Seed + 1 at int.MaxValue)
        sub = self._MBIG if seed == -2**31 else abs(seed)
        a = [0] * 56
        mj = self._sub(self._MSEED, sub)
        a[55] = mj
        mk = 1
        for i in range(1, 55):
            ii = (21 * i) % 55
            a[ii] = mk
            mk = self._sub(mj, mk)
            if mk < 0:
                mk += self._MBIG
            mj = a[ii]
        for _ in range(4):
            for i in range(1, 56):
                v = self._sub(a[i], a[1 + (i + 30) % 55])
                if v < 0:
                    v += self._MBIG
                a[i] = v
        self._a = a
        self._inext = 0
        self._inextp = 21

    def next(self) -> int:
        """Random.Next(): a value in [0, 2^31 - 1)."""
        self._inext = 1 if self._inext + 1 >= 56 else self._inext + 1
        self._inextp = 1 if self._inextp + 1 >= 56 else self._inextp + 1
        v = self._sub(self._a[self._inext], self._a[self._inextp])
        if v == self._MBIG:
            v -= 1
        if v < 0:
            v += self._MBIG
        self._a[self._inext] = v
        return v

    def next_double(self) -> float:
        """Random.NextDouble()."""
        return self.next() * (1.0 / self._MBIG)
