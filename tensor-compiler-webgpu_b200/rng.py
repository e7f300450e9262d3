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
    _CHUNK = 1 << 22   # draws per block: temporaries stay a few MB however many draws are asked for

    @staticmethod
    def _hash_array(t):
        """The mulberry32 output hash of uint32 states ``t`` (numpy's uint32 arithmetic wraps mod 2**32,
        as Math.imul and >>> 0 do)."""
        t = (t ^ (t >> np.uint32(15))) * (t | np.uint32(1))
        t = t ^ (t + (t ^ (t >> np.uint32(7))) * (t | np.uint32(61)))
        return t ^ (t >> np.uint32(14))

    def _states(self, k0, n):
        """The states of draws k0 + 1 .. k0 + n after the current one (uint32)."""
        k = np.arange(k0 + 1, k0 + n + 1, dtype=np.uint64) & np.uint64(_M32)
        return (np.uint32(self.state) + k.astype(np.uint32) * np.uint32(_STEP)).astype(np.uint32)

    def _uniforms(self, k0, n):
        """Uniforms of draws k0 + 1 .. k0 + n after the current one, as float64 (the state is unchanged)."""
        with np.errstate(over="ignore"):
            return self._hash_array(self._states(k0, n)) * (1.0 / 4294967296.0)

    @staticmethod
    def _blocks(n, block, fill):
        """Run ``fill(j0, m)`` over [0, n) in blocks of ``block``, on the host's cores when there are many
        (numpy releases the interpreter lock inside its loops; every block writes its own slice)."""
        starts = list(range(0, n, block))
        if len(starts) <= 2:
            for j0 in starts:
                fill(j0, min(block, n - j0))
            return
        from concurrent.futures import ThreadPoolExecutor
        import os
        with ThreadPoolExecutor(max_workers=min(len(starts), os.cpu_count() or 1, 32)) as ex:
            list(ex.map(lambda j0: fill(j0, min(block, n - j0)), starts))

    def next_array(self, n):
        """The next ``n`` uniforms in [0, 1) as float64, advancing the state by ``n``."""
        out = np.empty(n, dtype=np.float64)

        def fill(k0, m):
            out[k0:k0 + m] = self._uniforms(k0, m)
        self._blocks(n, self._CHUNK, fill)
        self.state = (self.state + n * _STEP) & _M32
        return out

    def uniform_array(self, n, lo, hi):
        return lo + (hi - lo) * self.next_array(n)

    def normal_array(self, n, mean=0.0, std=1.0):
        """Box-Muller over consecutive uniform pairs (u1, u2): one normal per pair."""
        out = np.empty(n, dtype=np.float64)

        def fill(j0, m):
            u = self._uniforms(2 * j0, 2 * m)
            u1, u2 = u[0::2], u[1::2]
            z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
            out[j0:j0 + m] = mean + std * z
        self._blocks(n, self._CHUNK // 2, fill)
        self.state = (self.state + 2 * n * _STEP) & _M32
        return out
