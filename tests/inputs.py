"""Seeded synthetic inputs for the parity tests and the bench (BASELINE.json
configs). A splitmix64 counter generator in numpy keeps the streams
independent of numpy's own RNG versions."""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


class Rng:
    def __init__(self, seed: int, stream: int = 0):
        self.key = int(_mix(np.array([seed * 1000003 + stream], np.uint64))[0])
        self.ctr = 0

    def bits(self, n: int) -> np.ndarray:
        i = np.arange(self.ctr, self.ctr + n, dtype=np.uint64)
        self.ctr += n
        with np.errstate(over="ignore"):
            return _mix(i * np.uint64(0x632BE59BD9B4E019) + np.uint64(self.key))

    def uniform(self, n: int, lo=0.0, hi=1.0) -> np.ndarray:
        u = (self.bits(n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
        return (lo + (hi - lo) * u).astype(np.float32)

    def normal(self, n: int, std=1.0) -> np.ndarray:
        m = (n + 1) // 2
        u1 = np.maximum((self.bits(m) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0), 1e-300)
        u2 = (self.bits(m) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
        r = np.sqrt(-2.0 * np.log(u1))
        z = np.empty(2 * m)
        z[0::2] = r * np.cos(2 * np.pi * u2)
        z[1::2] = r * np.sin(2 * np.pi * u2)
        return (z[:n] * std).astype(np.float32)

    def ints(self, n: int, hi: int) -> np.ndarray:
        return (self.bits(n) % np.uint64(hi)).astype(np.uint32)


def to_chain_major(cache: np.ndarray) -> np.ndarray:
    """[2][cap][256] position order -> [2][64][cap/64][256] (position p at chain p%64, slot p/64)."""
    h, cap, d = cache.shape
    return np.ascontiguousarray(cache.reshape(h, cap // 64, 64, d).transpose(0, 2, 1, 3))


def from_chain_major(cache: np.ndarray) -> np.ndarray:
    h, c, s, d = cache.reshape(cache.shape[0], 64, -1, cache.shape[-1]).shape
    return np.ascontiguousarray(cache.reshape(h, 64, s, d).transpose(0, 2, 1, 3).reshape(h, s * 64, d))


def f2bf(x) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf2f(h) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def pack_q4(q: np.ndarray) -> np.ndarray:
    """q [N, K] ints 0..15 -> codes [N, K/8] u32 (nibble k at bits 4*(k%8))."""
    n, k = q.shape
    q = q.astype(np.uint32).reshape(n, k // 8, 8)
    w = np.zeros((n, k // 8), np.uint32)
    for t in range(8):
        w |= q[:, :, t] << np.uint32(4 * t)
    return w


def unpack_q4(w: np.ndarray) -> np.ndarray:
    n, kw = w.shape
    q = np.zeros((n, kw, 8), np.uint32)
    for t in range(8):
        q[:, :, t] = (w >> np.uint32(4 * t)) & np.uint32(15)
    return q.reshape(n, kw * 8)


def config1(seed: int = 0, n: int = 3584, k: int = 1024):
    """W n x k, codes U{0..15}, per-64 scale ~U(0.005,0.02), bias = -8*scale,
    x ~ N(0,1) bf16."""
    r = Rng(seed, 1)
    q = r.ints(n * k, 16).reshape(n, k)
    scale = f2bf(r.uniform(n * (k // 64), 0.005, 0.02)).reshape(n, k // 64)
    bias = f2bf(-8.0 * bf2f(scale))
    x = f2bf(r.normal(k))
    return pack_q4(q), scale, bias, x


def config2(seed: int = 1):
    """one GDN decode step (16 heads, 128/128) with the gated out_proj."""
    r = Rng(seed, 2)
    d = {}
    d["raw"] = f2bf(r.normal(6144))
    d["z"] = f2bf(r.normal(2048))
    d["a"] = f2bf(r.normal(16))
    d["b"] = f2bf(r.normal(16))
    d["hist"] = f2bf(r.normal(3 * 6144))
    d["conv_w"] = f2bf(r.normal(6144 * 4, 0.3))
    d["a_log"] = r.uniform(16, -1.0, 1.0)
    d["dt"] = f2bf(r.uniform(16, -1.0, 1.0))
    d["state"] = r.normal(16 * 128 * 128, 0.05)
    d["norm_w"] = f2bf(1.0 + r.normal(128, 0.02))
    ow, os_, ob, _ = config1(seed + 100, 1024, 2048)
    d["ow"], d["os"], d["ob"] = ow, os_, ob
    d["res"] = f2bf(r.normal(1024))
    return d


def config3(seed: int = 2, length: int = 32768, capacity: int | None = None):
    """gated GQA decode at context `length` (8 q / 2 kv heads, D 256)."""
    cap = capacity or ((length + 63) // 64) * 64
    r = Rng(seed, 3)
    d = {}
    d["q_raw"] = f2bf(r.normal(4096))
    d["k_raw"] = f2bf(r.normal(512))
    d["v_raw"] = f2bf(r.normal(512))
    d["q_gain"] = f2bf(1.0 + r.normal(256, 0.02))
    d["k_gain"] = f2bf(1.0 + r.normal(256, 0.02))
    kc = np.zeros((2, cap, 256), np.uint16)
    vc = np.zeros((2, cap, 256), np.uint16)
    n_prev = length - 1
    if n_prev > 0:
        kc[:, :n_prev] = f2bf(r.normal(2 * n_prev * 256)).reshape(2, n_prev, 256)
        vc[:, :n_prev] = f2bf(r.normal(2 * n_prev * 256)).reshape(2, n_prev, 256)
    d["kc"], d["vc"], d["cap"], d["pos"] = kc, vc, cap, length - 1
    return d
