"""mulberry32, bit-exact with ``src/testing/rng.js:4-32``, plus vectorised draws.

mulberry32's state advances by a constant, so draw ``k`` (0-based) of a stream
seeded ``s`` depends only on ``s + (k + 1) * 0x6D2B79F5 mod 2**32``; the numpy
form evaluates that hash for many ``k`` at once and gives the same numbers as
the scalar form, draw for draw.

The reference has no normal sampler.  ``normal`` here is Box-Muller over two
consecutive uniforms ``u1, u2``: ``sqrt(-2 ln(1 - u1)) * cos(2 pi u2)``, one
normal per pair, the sine half discarded.
"""
from __future__ import annotations

import math

import numpy as np

_M32 = 0xFFFFFFFF
_STEP = 0x6D2B79F5


def _imul(a, b):
    return (a * b) & _M32


def _hash(t):
    t = _imul(t ^ (t >> 15), t | 1)
    t ^= (t + _imul(t ^ (t >> 7), t | 61)) & _M32
    return (t ^ (t >> 14)) & _M32


class Rng:
    """src/testing/rng.js:4-32."""

    def __init__(self, seed):
        self.state = seed & _M32

    def next(self):
        self.state = (self.state + _STEP) & _M32
        return _hash(self.state) / 4294967296.0

    def int(self, lo, hi):
        return lo + math.floor(self.next() * (hi - lo + 1))

    def uniform(self, lo, hi):
        return lo + (hi - lo) * self.next()

    def pick(self, items):
        return items[math.floor(self.next() * len(items))]

    def chance(self, p):
        return self.next() < p

    def array(self, n, lo=-1.0, hi=1.0):
        return [self.uniform(lo, hi) for _ in range(n)]

    def shuffle(self, items):
        a = list(items)
        for i in range(len(a) - 1, 0, -1):
            j = math.floor(self.next() * (i + 1))
            a[i], a[j] = a[j], a[i]
        return a

    # ---- vectorised draws (same stream, many draws at once) ----
    def next_array(self, n):
        """The next ``n`` uniforms in [0, 1) as float64, advancing the state by ``n``."""
        k = np.arange(1, n + 1, dtype=np.uint64)
        t = ((np.uint64(self.state) + k * np.uint64(_STEP)) & np.uint64(_M32)).astype(np.uint32)
        self.state = (self.state + n * _STEP) & _M32
        t = t.astype(np.uint64)
        m = np.uint64(_M32)
        a = t ^ (t >> np.uint64(15))
        t = (a * (t | np.uint64(1))) & m
        b = t ^ (t >> np.uint64(7))
        t = t ^ ((t + ((b * (t | np.uint64(61))) & m)) & m)
        t = (t ^ (t >> np.uint64(14))) & m
        return t.astype(np.float64) / 4294967296.0

    def uniform_array(self, n, lo, hi):
        return lo + (hi - lo) * self.next_array(n)

    def normal_array(self, n, mean=0.0, std=1.0):
        u = self.next_array(2 * n)
        u1, u2 = u[0::2], u[1::2]
        z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
        return mean + std * z
