"""The reference test suites' deterministic PRNGs, restated for fixtures.

* ``xs32`` / ``pseudo_i8``: src/simd/scalar.rs tests and dispatch.rs:340-349.
* ``Xs64``: tests/int4_packed_parity.rs, tests/lmhead_shard_parity.rs,
  tests/batched_igemm_parity.rs (x ^= x<<13; x ^= x>>7; x ^= x<<17).
"""
import numpy as np

M32 = 0xFFFFFFFF
M64 = 0xFFFFFFFFFFFFFFFF


def xs32_stream(seed, n):
    s = seed & M32
    out = np.empty(n, np.uint32)
    for i in range(n):
        s ^= (s << 13) & M32
        s ^= s >> 17
        s ^= (s << 5) & M32
        out[i] = s
    return out, s


def pseudo_i8(n, seed):
    v, _ = xs32_stream(seed | 1, n)
    return (v & 0xFF).astype(np.uint8).view(np.int8)


def pseudo_u8(n, seed):
    v, _ = xs32_stream(seed | 1, n)
    return (v & 0xFF).astype(np.uint8)


def rotl32(x, r):
    return ((x << r) | (x >> (32 - r))) & M32


class Xs64:
    def __init__(self, state):
        self.s = state & M64

    def next(self):
        x = self.s
        x ^= (x << 13) & M64
        x ^= x >> 7
        x ^= (x << 17) & M64
        self.s = x
        return x

    def fill_i8q(self, n):  # int4_packed_parity.rs Rng::i8q: (next % 255) - 127
        return np.array([(self.next() % 255) - 127 for _ in range(n)], np.int8)

    def fill_bytes(self, n):
        return np.array([self.next() & 0xFF for _ in range(n)], np.uint8)

    def fill_scales(self, n):  # ((next % 4096)/4096 - 0.5) * 1.7 in f32
        out = np.empty(n, np.float32)
        for i in range(n):
            v = np.float32(self.next() % 4096) / np.float32(4096.0)
            out[i] = (v - np.float32(0.5)) * np.float32(1.7)
        return out

    def fill_i8(self, n):  # lmhead/batched parity Rng::i8: next & 0xff
        return np.array([self.next() & 0xFF for _ in range(n)], np.uint8).view(np.int8)
