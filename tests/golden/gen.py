"""Portable input generator for the golden fixtures.

The fixtures under tests/golden/ hold only the reference's outputs; the inputs are rebuilt
here from a seed with splitmix64 in plain uint64 arithmetic, so they do not depend on
numpy's Generator streams.  Byte layouts follow GGUF Q4_K (144 B) / Q6_K (210 B) / Q8_0 (34 B)
blocks with the same field fix-ups as dracomancer_llmengine_b200.synth.
"""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n pseudo-random uint64 words from `seed` (Steele, Lea, Flood: SplitMix64)."""
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def rand_bytes(seed: int, n: int) -> np.ndarray:
    w = splitmix64(seed, (n + 7) // 8)
    return w.view(np.uint8)[:n].copy()


def rand_uniform(seed: int, n: int) -> np.ndarray:
    """float32 in [-1, 1) from the top 24 bits of each word."""
    w = splitmix64(seed, n) >> np.uint64(40)
    return (w.astype(np.float64) / float(1 << 23) - 1.0).astype(np.float32)


def q4k(seed: int, nblk: int) -> np.ndarray:
    b = rand_bytes(seed, nblk * 144).reshape(nblk, 144)
    r = rand_bytes(seed + 1, nblk * 8).reshape(nblk, 8).astype(np.int32)
    sc = 8 + r % 56
    mn = np.clip(np.rint(7.5 * sc / 8.0), 0, 63).astype(np.int32)
    d = (0.02 / (4.61 * sc.mean(axis=1))).astype(np.float16)
    dmin = (8.0 * d.astype(np.float32)).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    b[:, 2:4] = dmin.view(np.uint8).reshape(nblk, 2)
    s = np.zeros((nblk, 12), np.int32)
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    b[:, 4:16] = s.astype(np.uint8)
    return b


def q6k(seed: int, nblk: int) -> np.ndarray:
    b = rand_bytes(seed, nblk * 210).reshape(nblk, 210)
    r = rand_bytes(seed + 1, nblk * 16).reshape(nblk, 16).astype(np.int32)
    mag = 16 + r % 112
    sc = np.where(r & 1, mag, -mag).astype(np.int8)
    b[:, 192:208] = sc.view(np.uint8)
    d = (0.02 / (18.5 * np.abs(sc.astype(np.float32)).mean(axis=1))).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(nblk, 2)
    return b


def q8_0(seed: int, nblk: int) -> np.ndarray:
    b = rand_bytes(seed, nblk * 34).reshape(nblk, 34)
    b[:, 0:2] = np.full(nblk, 0.02 / 73.0, np.float32).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    q = b[:, 2:34].view(np.int8)
    q[q == -128] = -127
    return b


GEN = {5: (q4k, 144, 256), 4: (q6k, 210, 256), 0: (q8_0, 34, 32)}


def matrix(seed: int, code: int, n_mat: int, n_out: int, n_in: int) -> np.ndarray:
    fn, bb, bv = GEN[code]
    return fn(seed, n_mat * n_out * (n_in // bv)).reshape(n_mat, -1)


class Layer:
    """Duck-typed like synth.MoELayer (what the oracle wrappers read)."""

    def __init__(self, seed, hidden, n_exp, n_used, inter, scoring="softmax", n_group=1, n_group_used=1,
                 norm_w=1, w_scale=0.0, bias=False, code_gu=5, code_d=4):
        self.hidden, self.n_exp, self.n_used, self.inter = hidden, n_exp, n_used, inter
        self.scoring, self.n_group, self.n_group_used = scoring, n_group, n_group_used
        self.norm_w, self.w_scale, self.code_gu, self.code_d = norm_w, w_scale, code_gu, code_d
        self.gate = matrix(seed * 16 + 1, code_gu, n_exp, inter, hidden)
        self.up = matrix(seed * 16 + 3, code_gu, n_exp, inter, hidden)
        self.down = matrix(seed * 16 + 5, code_d, n_exp, hidden, inter)
        self.gate_inp = (rand_uniform(seed * 16 + 7, n_exp * hidden) * np.float32(0.05)).reshape(n_exp, hidden)
        self.probs_b = (rand_uniform(seed * 16 + 9, n_exp) * np.float32(0.02)) if bias else None
        self.shared_inter = 0

    def ptr_table(self):
        E = self.n_exp
        ep = np.zeros(3 * E, np.uint64)
        ec = np.zeros(3 * E, np.int32)
        for idx, (buf, code) in enumerate(((self.gate, self.code_gu), (self.up, self.code_gu),
                                           (self.down, self.code_d))):
            ep[idx::3] = buf.ctypes.data + buf.shape[1] * np.arange(E, dtype=np.uint64)
            ec[idx::3] = code
        return ep, ec


def tokens(seed: int, t: int, h: int) -> np.ndarray:
    x = rand_uniform(seed * 16 + 11, t * h).reshape(t, h) * np.float32(1.7)
    return (x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)


# fixture cases: name -> (layer kwargs, tokens)
CASES = {
    "granite_decode": (dict(seed=1, hidden=256, n_exp=4, n_used=2, inter=256), 3),
    "bailing_groups": (dict(seed=2, hidden=256, n_exp=8, n_used=2, inter=256, scoring="sigmoid", n_group=4,
                            n_group_used=2, w_scale=2.5, bias=True), 3),
    "bailing_k2style": (dict(seed=3, hidden=512, n_exp=4, n_used=3, inter=256, scoring="sigmoid", w_scale=2.827,
                             bias=True, code_d=0), 2),
}
