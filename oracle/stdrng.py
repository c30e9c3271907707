"""Restatement of the C++ standard-library random draws the reference's seeded initialisation uses.

TEST INFRASTRUCTURE ONLY (the checker of the library's seeded init; never imported by the product).

init_train_lora_state (src/train_lora.h:205-273) draws every target's A, target after target, as
std::uniform_real_distribution<float>(-1/sqrt(in), 1/sqrt(in)) from one std::mt19937_64(seed).
  mt19937_64       the 64-bit Mersenne Twister of Matsumoto and Nishimura (2004) with the
                   parameters the C++ standard fixes for std::mt19937_64 ([rand.predef]); pinned by
                   the standard's known answer: the 10000th output of a default-seeded engine is
                   9981545732273789042
  canonical float  libstdc++'s generate_canonical<float, 24> over a 64-bit engine: one draw x,
                   the float nearest x (round to nearest even) divided by 2^64, 1 mapped to the
                   largest float below 1
  uniform float    (b - a) * u + a in float arithmetic
"""
import math

import numpy as np

_N, _M = 312, 156
_MATRIX_A = 0xB5026F5AA96619E9
_UPPER, _LOWER = 0xFFFFFFFF80000000, 0x7FFFFFFF
_MASK = (1 << 64) - 1


class MT19937_64:
    def __init__(self, seed=5489):
        mt = [0] * _N
        mt[0] = seed & _MASK
        for i in range(1, _N):
            mt[i] = (6364136223846793005 * (mt[i - 1] ^ (mt[i - 1] >> 62)) + i) & _MASK
        self.mt, self.i = mt, _N

    def _twist(self):
        mt = self.mt
        for i in range(_N):
            x = (mt[i] & _UPPER) | (mt[(i + 1) % _N] & _LOWER)
            xa = x >> 1
            if x & 1:
                xa ^= _MATRIX_A
            mt[i] = mt[(i + _M) % _N] ^ xa
        self.i = 0

    def __call__(self):
        if self.i >= _N:
            self._twist()
        x = self.mt[self.i]
        self.i += 1
        x ^= (x >> 29) & 0x5555555555555555
        x ^= (x << 17) & 0x71D67FFFEDA60000
        x ^= (x << 37) & 0xFFF7EEE000000000
        x ^= x >> 43
        return x & _MASK


def _u64_to_f32(x):
    """The float nearest the integer x (round half to even), exactly."""
    if x == 0:
        return np.float32(0.0)
    e = x.bit_length() - 24
    if e <= 0:
        return np.float32(x)
    q, r = divmod(x, 1 << e)
    half = 1 << (e - 1)
    if r > half or (r == half and q & 1):
        q += 1
    return np.float32(math.ldexp(q, e))


def canonical_float(eng):
    u = np.float32(_u64_to_f32(eng()) / np.float32(2.0 ** 64))
    if u >= np.float32(1.0):
        u = np.nextafter(np.float32(1.0), np.float32(0.0))
    return u


def uniform_float(eng, a, b):
    a, b = np.float32(a), np.float32(b)
    return np.float32(np.float32(canonical_float(eng) * np.float32(b - a)) + a)


def lora_init_A(seed, targets, rank):
    """A of every target (list of (in, out)) in order, as init_train_lora_state draws them."""
    eng = MT19937_64(seed)
    out = []
    for inn, _ in targets:
        bound = np.float32(np.float32(1.0) / np.sqrt(np.float32(inn)))
        out.append(np.array([uniform_float(eng, -bound, bound) for _ in range(rank * inn)], np.float32))
    return out
