"""The CPU oracle pinned against the reference: golden fixtures (made from the reference's own
C by tests/golden/make_golden.py), the live reference build in oracle/_ref when present, the
third-party gguf-py decoder, and known-answer tests for the Q8_K restatement."""
import os
import re
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import gen  # noqa: E402
from dracomancer_llmengine_b200 import synth  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ----------------------------------------------------------------------------- fixtures
@pytest.mark.parametrize("name", list(gen.CASES))
def test_port_matches_golden_fixtures(port, name):
    kw, T = gen.CASES[name]
    layer = gen.Layer(**kw)
    X = gen.tokens(kw["seed"], T, layer.hidden)
    g = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    # decode layer, gemv rows: bit-identical to the reference's C
    assert np.array_equal(bits(port.decode(layer, X)), bits(g["decode"]))
    assert np.array_equal(bits(port.gemv(layer.code_gu, X[0], layer.gate[0], layer.inter, layer.hidden)),
                          bits(g["gemv_gate"]))
    assert np.array_equal(bits(port.gemv(layer.code_d, X[0][:layer.inter].copy(), layer.down[0], layer.hidden,
                                         layer.inter)), bits(g["gemv_down"]))
    # chunked prefill: the reference sums 16 lanes at a time, the oracle row by row
    tok = port.moe_tok(layer, X, g["order"], g["wtop"])
    rel = np.linalg.norm(tok - g["moe_tok"]) / np.linalg.norm(g["moe_tok"])
    assert rel < 1e-6, rel


def test_fixture_inputs_are_stable():
    # the generator is plain integer arithmetic: pin a few words so a change is noticed
    w = gen.splitmix64(0, 3)
    assert [int(v) for v in w] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


# ----------------------------------------------------------------------------- live reference
CASES_LIVE = {
    "granite_e32": dict(hidden=2048, n_exp=32, n_used=8, inter=768, seed=5),
    "granite_k6": dict(hidden=1024, n_exp=16, n_used=6, inter=512, seed=6),
    "bailing_groups": dict(hidden=2048, n_exp=32, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                           n_group_used=4, w_scale=2.5, bias=True, seed=7),
    "k2_shape": dict(hidden=7168, n_exp=16, n_used=8, inter=2048, scoring="sigmoid", w_scale=2.827, bias=True,
                     seed=8),
}


@pytest.mark.parametrize("name", list(CASES_LIVE))
def test_port_bitexact_with_reference_decode(port, ref, name):
    layer = synth.make_layer(**CASES_LIVE[name])
    X = synth.make_tokens(layer, 3, CASES_LIVE[name]["seed"])
    assert np.array_equal(bits(port.decode(layer, X)), bits(ref.decode(layer, X)))


@pytest.mark.parametrize("code,n_out,n_in", [(5, 64, 2048), (4, 64, 768), (4, 32, 2048), (0, 48, 512)])
def test_port_bitexact_with_reference_gemv(port, ref, code, n_out, n_in):
    rng = np.random.default_rng(code + n_in)
    W = synth.quant_matrix(rng, code, 1, n_out, n_in)[0]
    x = rng.standard_normal(n_in).astype(np.float32)
    assert np.array_equal(bits(port.gemv(code, x, W, n_out, n_in)), bits(ref.gemv(code, x, W, n_out, n_in)))


def test_port_moe_tok_with_reference(port, ref):
    layer = synth.make_layer(hidden=2048, n_exp=16, n_used=4, inter=512, seed=9)
    X = synth.make_tokens(layer, 24, 9)
    order, wtop = port.route(layer, X)
    a = port.moe_tok(layer, X, order, wtop)
    b = ref.moe_tok(layer, X, order, wtop, fused=True)
    c = ref.moe_tok(layer, X, order, wtop, fused=False)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-6
    assert np.array_equal(b, c)       # the reference's two prefill paths agree bit for bit


def test_port_moe_tok_equals_decode(port):
    """Prefill and per-token decode are the same function of the routing (the reference's
    prefill-vs-decode gate, tests/prefill_chunk_gate.py); they differ only in how the combine
    rounds (decode: products rounded then summed, prefill: fused multiply-adds)."""
    layer = synth.make_layer(hidden=1024, n_exp=16, n_used=4, inter=512, seed=10)
    X = synth.make_tokens(layer, 5, 10)
    order, wtop = port.route(layer, X)
    a, b = port.moe_tok(layer, X, order, wtop), port.decode(layer, X)
    assert np.abs(a - b).max() <= 4 * np.finfo(np.float32).eps * np.abs(b).max()


def test_gemvn_reference_redundant_rows_but_same_values(port, ref):
    """m5_gemvn_q4k recomputes every row per 96-row block (a reference bug that only costs
    time); its values still equal per-expert gemv to fp32 summation order."""
    rng = np.random.default_rng(12)
    E, n_out, n_in = 6, 200, 1024
    W = synth.quant_matrix(rng, 5, E, n_out, n_in)
    idx = np.array([3, 1, 5], np.int32)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = ref.gemvn(5, x, 0, W, idx, W.shape[1], n_out, n_in)
    exp = np.concatenate([port.gemv(5, x, W[e], n_out, n_in) for e in idx])
    assert np.abs(y - exp).max() < 1e-4 * np.abs(exp).max()


# ----------------------------------------------------------------------------- gguf-py
def test_dequant_matches_gguf_py(port):
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(13)
    for code, gt, n_in in ((5, gguf.GGMLQuantizationType.Q4_K, 512), (4, gguf.GGMLQuantizationType.Q6_K, 512),
                           (0, gguf.GGMLQuantizationType.Q8_0, 256)):
        W = synth.quant_matrix(rng, code, 1, 8, n_in)[0]
        ours = port.dequant(code, W, 8, n_in)
        theirs = np.asarray(gguf.quants.dequantize(W, gt), np.float32).reshape(8, n_in)
        assert np.allclose(ours, theirs, rtol=2e-7, atol=1e-9), code


def test_synth_distribution():
    rng = np.random.default_rng(14)
    for code in (5, 4, 0):
        from oracle.oracle import Port
        W = synth.quant_matrix(rng, code, 1, 64, 512)[0]
        v = Port().dequant(code, W, 64, 512)
        assert 0.015 < float(np.sqrt((v ** 2).mean())) < 0.03
        assert abs(float(v.mean())) < 2e-3


def test_zipf_router_is_skewed(port):
    layer, X = synth.make_config("cfg5_k2_prefill_zipf", tokens=64, weights=False)
    # router only: cheap at 64 tokens
    idx, _ = port.route(layer, X)
    counts = np.bincount(idx.ravel(), minlength=layer.n_exp)
    top = np.sort(counts)[::-1]
    assert top[:8].sum() > 0.25 * counts.sum()      # hot experts dominate
    uni_layer, uX = synth.make_config("cfg3_k2_decode", tokens=64, weights=False)
    uidx, _ = port.route(uni_layer, uX)
    ucounts = np.sort(np.bincount(uidx.ravel(), minlength=384))[::-1]
    assert top[:8].sum() > 2 * ucounts[:8].sum()


# ----------------------------------------------------------------------------- Q8_K known answers
def test_q8k_quantize_known_answers(port):
    x = np.zeros(512, np.float32)
    x[0], x[1], x[2], x[3] = 2.0, -1.0, 0.5, 1.0      # amax 2 -> d = 2/127, q = rint(x * 63.5)
    x[300] = -4.0                                     # second block: only one non-zero value
    d, q, bs = port.q8k_quantize(x)
    assert d[0] == np.float32(1.0) / (np.float32(127.0) / np.float32(2.0))
    assert list(q[:4]) == [127, -64, 32, 64]          # rint(-63.5) = -64, rint(31.75) = 32
    assert bs[0] == 127 - 64 + 32 + 64
    assert q[300] == -127 and bs[16 + (300 - 256) // 16] == -127
    z = np.zeros(256, np.float32)
    d0, q0, b0 = port.q8k_quantize(z)
    assert d0[0] == 0 and not q0.any() and not b0.any()


def test_q4k_q8k_block_known_answer(port):
    # all nibbles = 3, sub-block scales 1..8, mins 0..7, q8 = 1 everywhere
    blk = np.zeros(144, np.uint8)
    sc = np.arange(1, 9)
    mn = np.arange(0, 8)
    s = np.zeros(12, np.int32)
    s[0:4] = sc[0:4] | ((sc[4:8] >> 4) << 6)
    s[4:8] = mn[0:4] | ((mn[4:8] >> 4) << 6)
    s[8:12] = (sc[4:8] & 15) | ((mn[4:8] & 15) << 4)
    blk[4:16] = s
    blk[16:] = 0x33
    q8 = np.ones(256, np.int8)
    bsums = np.full(16, 16, np.int16)
    import ctypes as ct
    a = np.zeros(1, np.int32)
    m = np.zeros(1, np.int32)
    port.L.orc_q4k_q8k_block(blk.ctypes.data_as(ct.POINTER(ct.c_uint8)), q8.ctypes.data_as(ct.POINTER(ct.c_int8)),
                             bsums.ctypes.data_as(ct.POINTER(ct.c_int16)), a.ctypes.data_as(ct.POINTER(ct.c_int32)),
                             m.ctypes.data_as(ct.POINTER(ct.c_int32)))
    assert a[0] == sum(int(j) * 3 * 32 for j in sc)      # sum_j sc_j * (3 * 32)
    assert m[0] == sum(int(j) * 32 for j in mn)          # sum_j m_j * 32


def test_q6k_q8k_block_known_answer(port):
    blk = np.zeros(210, np.uint8)
    blk[0:128] = 0x11            # nibbles 1
    blk[128:192] = 0xAA          # 2-bit fields 2 -> q6 = 1 | 2<<4 = 33 -> 33 - 32 = 1
    blk[192:208] = np.arange(-8, 8, dtype=np.int8).view(np.uint8)
    q8 = np.full(256, 2, np.int8)
    import ctypes as ct
    out = np.zeros(1, np.int32)
    port.L.orc_q6k_q8k_block(blk.ctypes.data_as(ct.POINTER(ct.c_uint8)), q8.ctypes.data_as(ct.POINTER(ct.c_int8)),
                             out.ctypes.data_as(ct.POINTER(ct.c_int32)))
    assert out[0] == sum(g * 16 * 1 * 2 for g in range(-8, 8))


def test_q8k_gemv_close_to_f32_reference(port):
    """Q8_K mode changes the activations by their int8 rounding only: the Q8_K dot equals the
    fp32 dot on the dequantised activations to fp32 rounding."""
    rng = np.random.default_rng(15)
    n_in, rows = 2048, 32
    x = synth.rms_normed(rng, 1, n_in)[0]
    d, q, bs = port.q8k_quantize(x)
    xhat = (q.reshape(-1, 256).astype(np.float32) * d[:, None]).reshape(-1)
    for code in (5, 4):
        W = synth.quant_matrix(rng, code, 1, rows, n_in)[0]
        y8 = port.gemv_q8k(code, d, q, bs, W, rows, n_in)
        yf = port.gemv(code, xhat, W, rows, n_in)
        assert np.abs(y8 - yf).max() < 1e-4 * max(1.0, np.abs(yf).max())


# ----------------------------------------------------------------------------- exp table
def test_device_exp_table_is_2_pow_i_over_32():
    mpmath = pytest.importorskip("mpmath")
    src = open(os.path.join(os.path.dirname(HERE), "dracomancer_llmengine_b200", "csrc", "common.cuh")).read()
    body = src[src.index("kExp2Tab[32]"):]
    vals = [int(v, 16) for v in re.findall(r"0x([0-9a-f]{16})ull", body)[:32]]
    mpmath.mp.prec = 200
    import struct
    for i, v in enumerate(vals):
        d = float(mpmath.mpf(2) ** (mpmath.mpf(i) / 32))
        u = struct.unpack("<Q", struct.pack("<d", d))[0]
        assert v == (u - (i << 47)) & 0xFFFFFFFFFFFFFFFF, i
