"""Seeded synthetic MoE layers in GGUF superblock formats.

No model files exist for this path, so every test and benchmark runs on weights drawn here
with the shapes of the configurations the engine is measured on.  The byte layouts are the
GGUF ones the reference decodes:

* Q4_K (code 5), 144 B per 256 values: fp16 d, fp16 dmin, 12 B of packed 6-bit (scale, min)
  pairs, 128 B of nibbles (`src/m5_kern_scalar.c:39-46,69-90` of the reference).
* Q6_K (code 4), 210 B per 256 values: ql[128], qh[64], int8 scales[16], fp16 d
  (`src/m5_kern_scalar.c:115-142`).
* Q8_0 (code 0), 34 B per 32 values: fp16 d, int8 q[32] (`src/m5_kern_scalar.c:58-68`).

Value distributions: dequantised weights have RMS ~0.02 and are centred (Q4_K's min term
cancels the nibble mean); router weights N(0, 0.02); expert bias N(0, 0.01); activations
N(0, 1) then RMS-normalised.  Zipf skew (alpha = 1.2, popularity permuted by the seed) is
put into the router logits through one hidden column that every token carries with the
same value, so the router itself produces the skewed logits.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np

CODE_Q8_0 = 0
CODE_Q6_K = 4
CODE_Q4_K = 5

BLOCK_BYTES = {CODE_Q8_0: 34, CODE_Q6_K: 210, CODE_Q4_K: 144}
BLOCK_VALUES = {CODE_Q8_0: 32, CODE_Q6_K: 256, CODE_Q4_K: 256}


def row_bytes(code: int, n_in: int) -> int:
    """Bytes of one weight row of `n_in` values (`src/m6_engine.c:40-54`)."""
    return (n_in // BLOCK_VALUES[code]) * BLOCK_BYTES[code]


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(v.astype(np.float16)).view(np.uint8).reshape(*v.shape, 2)


def _random_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniform random bytes (the generator's raw 64-bit outputs, little-endian)."""
    return rng.bit_generator.random_raw((n + 7) // 8).view(np.uint8)[:n]


def q4k_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    """`n` Q4_K superblocks, uint8 [n, 144]."""
    sc = rng.integers(8, 64, size=(n, 8), dtype=np.int32)
    mn = np.clip(np.rint(7.5 * sc / 8.0), 0, 63).astype(np.int32)
    d = (0.02 / (4.61 * sc.mean(axis=1))).astype(np.float16)
    dmin = (8.0 * d.astype(np.float32)).astype(np.float16)
    out = np.empty((n, 144), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    s = np.zeros((n, 12), np.int32)
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    out[:, 4:16] = s.astype(np.uint8)
    out[:, 16:144] = _random_bytes(rng, n * 128).reshape(n, 128)   # uniform nibbles
    return out


def q6k_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    """`n` Q6_K superblocks, uint8 [n, 210]."""
    out = np.empty((n, 210), np.uint8)
    out[:, 0:192] = _random_bytes(rng, n * 192).reshape(n, 192)   # uniform ql/qh bits
    mag = rng.integers(16, 128, size=(n, 16), dtype=np.int32)
    sgn = np.where(rng.integers(0, 2, size=(n, 16)) == 0, -1, 1)
    sc = (mag * sgn).astype(np.int8)
    out[:, 192:208] = sc.view(np.uint8)
    d = (0.02 / (18.5 * np.abs(sc.astype(np.float32)).mean(axis=1))).astype(np.float16)
    out[:, 208:210] = _f16_bytes(d)
    return out


def q8_0_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    """`n` Q8_0 blocks, uint8 [n, 34]."""
    q = rng.integers(-127, 128, size=(n, 32), dtype=np.int32).astype(np.int8)
    d = np.full(n, 0.02 / 73.0, np.float32).astype(np.float16)
    out = np.empty((n, 34), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:34] = q.view(np.uint8)
    return out


_GEN = {CODE_Q4_K: q4k_blocks, CODE_Q6_K: q6k_blocks, CODE_Q8_0: q8_0_blocks}


def quant_matrix(rng: np.random.Generator, code: int, n_mat: int, n_out: int, n_in: int) -> np.ndarray:
    """`n_mat` stacked [n_out x n_in] matrices, uint8 [n_mat, n_out * row_bytes]."""
    nb = n_in // BLOCK_VALUES[code]
    blocks = _GEN[code](rng, n_mat * n_out * nb)
    return blocks.reshape(n_mat, n_out * nb * BLOCK_BYTES[code])


def expert_matrices(seed, code: int, n_mat: int, n_out: int, n_in: int, first: int = 0) -> np.ndarray:
    """Like quant_matrix, with matrix e drawn from its own stream default_rng([*seed, e]), so the
    experts are generated in parallel (threads; numpy releases the GIL) and still reproducibly;
    `first` > 0 generates matrices first .. first + n_mat - 1 of the same sequence."""
    import concurrent.futures
    nb = n_in // BLOCK_VALUES[code]
    per = n_out * nb * BLOCK_BYTES[code]
    out = np.empty((n_mat, per), np.uint8)

    def one(e):
        out[e] = _GEN[code](np.random.default_rng([*seed, first + e]), n_out * nb).reshape(per)

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(one, range(n_mat)))
    return out


def rms_normed(rng: np.random.Generator, t: int, h: int) -> np.ndarray:
    x = rng.standard_normal((t, h), dtype=np.float32)
    return (x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)


@dataclasses.dataclass
class MoELayer:
    """One synthetic MoE FFN layer.  Stacked expert tensors use the GGUF layout
    (`base + e * per`, `src/qwen35_engine.py:243-248` of the reference)."""
    n_exp: int
    n_used: int
    inter: int
    hidden: int
    gate: np.ndarray            # uint8 [n_exp, inter * rb(code_gu, hidden)]
    up: np.ndarray
    down: np.ndarray            # uint8 [n_exp, hidden * rb(code_d, inter)]
    gate_inp: np.ndarray        # fp32 [n_exp, hidden]
    code_gu: int = CODE_Q4_K
    code_d: int = CODE_Q6_K
    scoring: str = "softmax"    # "softmax" | "sigmoid"
    probs_b: np.ndarray | None = None
    n_group: int = 1
    n_group_used: int = 1
    norm_w: int = 1
    w_scale: float = 0.0
    shared_inter: int = 0
    sh_gate: np.ndarray | None = None   # uint8 [shared_inter * rb]
    sh_up: np.ndarray | None = None
    sh_down: np.ndarray | None = None
    sh_gate_inp: np.ndarray | None = None  # fp32 [hidden] scalar-gated shared expert, or None
    expert0: int = 0            # gate/up/down hold experts expert0 .. expert0 + len - 1 (an
                                # expert-parallel rank's slice); all n_exp when 0 and full

    def ptr_table(self):
        """(ep uint64[3E], ec int32[3E]) host pointer table as the reference drivers build it;
        entries of experts this layer object does not hold are 0."""
        E = self.n_exp
        ep = np.zeros(3 * E, np.uint64)
        ec = np.zeros(3 * E, np.int32)
        for idx, (buf, code) in enumerate(((self.gate, self.code_gu), (self.up, self.code_gu),
                                           (self.down, self.code_d))):
            base = buf.ctypes.data
            per = buf.shape[1]
            n = buf.shape[0]
            ep[3 * self.expert0 + idx:3 * (self.expert0 + n):3] = base + per * np.arange(n, dtype=np.uint64)
            ec[idx::3] = code
        return ep, ec


CONFIGS = {
    # name: (hidden, n_exp, n_used, inter, tokens, scoring, n_group, n_group_used, w_scale,
    #        shared_inter, bias, zipf, seed)
    "cfg1_decode": dict(hidden=2048, n_exp=128, n_used=8, inter=768, tokens=1, scoring="softmax",
                        n_group=1, n_group_used=1, w_scale=0.0, shared_inter=0, bias=False,
                        zipf=False, seed=0),
    "cfg2_prefill": dict(hidden=2048, n_exp=128, n_used=8, inter=768, tokens=512, scoring="softmax",
                         n_group=1, n_group_used=1, w_scale=0.0, shared_inter=0, bias=False,
                         zipf=False, seed=1),
    "cfg3_k2_decode": dict(hidden=7168, n_exp=384, n_used=8, inter=2048, tokens=64, scoring="sigmoid",
                           n_group=1, n_group_used=1, w_scale=2.827, shared_inter=2048, bias=True,
                           zipf=False, seed=2),
    "cfg4_ling_prefill": dict(hidden=2048, n_exp=256, n_used=8, inter=512, tokens=4096,
                              scoring="sigmoid", n_group=8, n_group_used=4, w_scale=2.5,
                              shared_inter=512, bias=True, zipf=False, seed=3),
    "cfg5_k2_prefill_zipf": dict(hidden=7168, n_exp=384, n_used=8, inter=2048, tokens=8192,
                                 scoring="sigmoid", n_group=1, n_group_used=1, w_scale=2.827,
                                 shared_inter=2048, bias=True, zipf=True, seed=4),
}

ZIPF_ALPHA = 1.2
ZIPF_COLUMN = 0      # hidden column that carries the per-expert popularity offset


def make_layer(hidden: int, n_exp: int, n_used: int, inter: int, scoring: str = "softmax",
               n_group: int = 1, n_group_used: int = 1, w_scale: float = 0.0,
               shared_inter: int = 0, bias: bool = False, zipf: bool = False, seed: int = 0,
               code_gu: int = CODE_Q4_K, code_d: int = CODE_Q6_K, weights: bool = True,
               experts: tuple | None = None, **_unused) -> MoELayer:
    """Expert weights, router and shared expert come from independent seeded streams, so
    `weights=False` (router only, empty expert tensors) routes exactly like the full layer, and
    `experts=(first, count)` (one expert-parallel rank's slice) holds exactly those experts of
    the full layer."""
    first, count = experts if experts else (0, n_exp)
    if weights:
        gate = expert_matrices((seed, 0, 0), code_gu, count, inter, hidden, first)
        up = expert_matrices((seed, 0, 1), code_gu, count, inter, hidden, first)
        down = expert_matrices((seed, 0, 2), code_d, count, hidden, inter, first)
    else:
        gate = up = down = np.zeros((n_exp, 0), np.uint8)
    rng = np.random.default_rng([seed, 1])
    gi = (rng.standard_normal((n_exp, hidden), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if zipf:
        ranks = np.arange(1, n_exp + 1, dtype=np.float64)
        p = ranks ** -ZIPF_ALPHA
        p /= p.sum()
        perm = rng.permutation(n_exp)
        logp = np.empty(n_exp, np.float64)
        logp[perm] = np.log(p)
        gi[:, ZIPF_COLUMN] = logp.astype(np.float32)
    probs_b = (rng.standard_normal(n_exp, dtype=np.float32) * np.float32(0.01)).astype(np.float32) if bias else None
    layer = MoELayer(n_exp=n_exp, n_used=n_used, inter=inter, hidden=hidden, gate=gate, up=up,
                     down=down, gate_inp=gi, code_gu=code_gu, code_d=code_d, scoring=scoring,
                     probs_b=probs_b, n_group=n_group, n_group_used=n_group_used, norm_w=1,
                     w_scale=w_scale, expert0=first if weights else 0)
    if shared_inter and weights:
        rng = np.random.default_rng([seed, 2])
        layer.shared_inter = shared_inter
        layer.sh_gate = quant_matrix(rng, code_gu, 1, shared_inter, hidden)[0]
        layer.sh_up = quant_matrix(rng, code_gu, 1, shared_inter, hidden)[0]
        layer.sh_down = quant_matrix(rng, code_d, 1, hidden, shared_inter)[0]
    return layer


def make_tokens(layer: MoELayer, tokens: int, seed: int, zipf: bool = False) -> np.ndarray:
    rng = np.random.default_rng(seed + 7919)
    x = rms_normed(rng, tokens, layer.hidden)
    if zipf:
        # one column carries the same value for every token, so logits += log p(e)
        x[:, ZIPF_COLUMN] = 1.0
    return x


def make_config(name: str, tokens: int | None = None, weights: bool = True, experts: tuple | None = None):
    """(layer, X) for a named configuration; `tokens` overrides the token count, `experts` =
    (first, count) generates only that slice of the expert weights."""
    c = dict(CONFIGS[name])
    layer = make_layer(weights=weights, experts=experts, **c)
    x = make_tokens(layer, c["tokens"] if tokens is None else tokens, c["seed"], c["zipf"])
    return layer, x
