"""Parity of the CUDA path (called through the C ABI) with the CPU oracle on seeded inputs.

Bars (from the task's contract):
  * routing: selected expert indices and gate weights bit-exact (ties -> lower index);
  * Q8_K activations x Q4_K/Q6_K: integer superblock dots bit-exact;
  * final fp32 layer output: relative L2 error <= 1e-3 (REL_L2_TOL below).
"""
import ctypes as ct

import numpy as np
import pytest

from dracomancer_llmengine_b200 import synth
import dracomancer_llmengine_b200 as dm

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ----------------------------------------------------------------------------- exp
def test_expf_matches_host_libm(dlib, port):
    rng = np.random.default_rng(11)
    pats = rng.integers(0, 2 ** 32, size=1 << 22, dtype=np.uint64).astype(np.uint32)
    dense = np.linspace(-110.0, 90.0, 1 << 21, dtype=np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, 88.72283, 88.72284, -103.97207, -103.97208,
                        -87.3, 1e-30, -1e-30, 1.0, -1.0], np.float32)
    x = np.concatenate([pats.view(np.float32), dense, special])
    x = x[~np.isnan(x)]
    y = np.empty_like(x)
    assert dlib.draco_b200_expf(x.ctypes.data_as(dm._f), y.ctypes.data_as(dm._f), x.size) == 0
    ref = port.expf(x)
    mism = np.nonzero(bits(y) != bits(ref))[0]
    assert mism.size == 0, f"{mism.size} mismatches, first x={x[mism[:4]]} gpu={y[mism[:4]]} host={ref[mism[:4]]}"


# ----------------------------------------------------------------------------- routers
ROUTER_CASES = {
    "softmax_e128": dict(hidden=2048, n_exp=128, n_used=8, inter=256, seed=21),
    "sigmoid_groups_e256": dict(hidden=2048, n_exp=256, n_used=8, inter=256, scoring="sigmoid", n_group=8,
                                n_group_used=4, w_scale=2.5, bias=True, seed=22),
    "sigmoid_k2_e384": dict(hidden=7168, n_exp=384, n_used=8, inter=256, scoring="sigmoid", w_scale=2.827,
                            bias=True, seed=23),
    "sigmoid_zipf_e384": dict(hidden=7168, n_exp=384, n_used=8, inter=256, scoring="sigmoid", w_scale=2.827,
                              bias=True, zipf=True, seed=24),
    "softmax_k1": dict(hidden=512, n_exp=16, n_used=1, inter=256, seed=25),
    "sigmoid_nonorm": dict(hidden=512, n_exp=64, n_used=6, inter=256, scoring="sigmoid", bias=True, seed=26),
    # the numpy K2 drivers' renormalisation (norm_w = 2: no clamp, numpy's pairwise sum order)
    "sigmoid_k2_driver_renorm": dict(hidden=7168, n_exp=384, n_used=8, inter=256, scoring="sigmoid", w_scale=2.827,
                                     bias=True, seed=28),
    "sigmoid_k2_driver_renorm_k12": dict(hidden=512, n_exp=96, n_used=12, inter=256, scoring="sigmoid",
                                         w_scale=2.5, bias=True, seed=29),
}


@pytest.mark.parametrize("name", list(ROUTER_CASES))
def test_router_bitexact(dlib, port, name):
    c = dict(ROUTER_CASES[name])
    zipf = c.pop("zipf", False)
    layer = synth.make_layer(zipf=zipf, **c)
    if name == "sigmoid_nonorm":
        layer.norm_w = 0
    if name.startswith("sigmoid_k2_driver"):
        layer.norm_w = 2
    X = synth.make_tokens(layer, 48, c["seed"], zipf=zipf)
    o_gpu, w_gpu = dm.route(layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(o_gpu, o_ref), f"index mismatch rows {np.nonzero((o_gpu != o_ref).any(1))[0][:8]}"
    assert np.array_equal(bits(w_gpu), bits(w_ref)), "gate weights differ in bits"


def logits_ref(X, W):
    """Sequential float32 sums of rounded products, k ascending (the reference's C order)."""
    X = np.asarray(X, np.float32)
    W = np.asarray(W, np.float32)
    acc = np.zeros((X.shape[0], W.shape[0]), np.float32)
    for k in range(X.shape[1]):
        acc = acc + np.multiply.outer(X[:, k], W[:, k])   # float32 product rounded, then float32 add
    return acc


# shapes reaching every logits kernel: the small-batch tiles (deep and shallow rings, partial last
# chunk, batches of 1-5 tokens), the register-tiled kernel for many tiles with 5, 6, 7 and 8 token
# rows a warp, the scalar fallback (width % 4 != 0)
@pytest.mark.parametrize("T,E,H", [(1, 128, 2048), (3, 384, 7168), (4, 60, 516), (5, 128, 2048), (48, 384, 1024),
                                   (300, 128, 512), (600, 128, 2048), (2400, 256, 256), (2400, 256, 260),
                                   (40, 64, 258), (512, 128, 2048), (64, 384, 7168), (100, 128, 2048),
                                   (33, 90, 1028), (4744, 128, 256), (5928, 128, 260), (7112, 128, 256),
                                   (4680, 128, 256), (2048, 256, 256), (1024, 384, 516)])
def test_router_logits_exact_order(dlib, T, E, H):
    rng = np.random.default_rng(T + E + H)
    X = rng.standard_normal((T, H), dtype=np.float32)
    W = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    got = np.empty((T, E), np.float32)
    assert dlib.draco_b200_router_logits(X.ctypes.data_as(dm._f), W.ctypes.data_as(dm._f), T, E, H,
                                         got.ctypes.data_as(dm._f)) == 0, dm.last_error()
    ref = logits_ref(X, W)
    bad = np.nonzero(bits(got) != bits(ref))
    assert bad[0].size == 0, f"{bad[0].size} logits differ, first (t, e) {list(zip(bad[0][:4], bad[1][:4]))}"


@pytest.mark.parametrize("name,T", [("softmax_e128", 600), ("sigmoid_groups_e256", 2400), ("sigmoid_k2_e384", 200)])
def test_router_bitexact_large_batches(dlib, port, name, T):
    """Token batches large enough for the register-tiled logits kernel."""
    c = dict(ROUTER_CASES[name])
    zipf = c.pop("zipf", False)
    layer = synth.make_layer(zipf=zipf, weights=False, **c)
    X = synth.make_tokens(layer, T, c["seed"] + 1, zipf=zipf)
    o_gpu, w_gpu = dm.route(layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(o_gpu, o_ref), f"index mismatch rows {np.nonzero((o_gpu != o_ref).any(1))[0][:8]}"
    assert np.array_equal(bits(w_gpu), bits(w_ref)), "gate weights differ in bits"


def test_router_ties_lower_index(dlib, port):
    layer = synth.make_layer(hidden=256, n_exp=32, n_used=8, inter=256, seed=27)
    # duplicate router rows: experts 2k and 2k+1 score identically -> ties everywhere
    layer.gate_inp[1::2] = layer.gate_inp[0::2]
    X = synth.make_tokens(layer, 16, 27)
    o_gpu, w_gpu = dm.route(layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(o_gpu, o_ref)
    assert np.array_equal(bits(w_gpu), bits(w_ref))
    # every tied pair is taken lower index first
    for row in o_gpu:
        for j, e in enumerate(row):
            if e % 2 == 1:
                assert e - 1 in row[:j]


def test_router_group_limit_error(dlib):
    # 2 groups of 4, only 1 group kept, but 6 experts wanted: the reference reads out of
    # bounds here; the device path refuses the shape
    layer = synth.make_layer(hidden=256, n_exp=8, n_used=6, inter=256, scoring="sigmoid", n_group=2,
                             n_group_used=1, bias=True, seed=28)
    with pytest.raises(dm.DracoError):
        dm.route(layer, synth.make_tokens(layer, 2, 28))


# ----------------------------------------------------------------------------- decode layers
def test_granite_moe_cfg1(dlib, port):
    layer, X = synth.make_config("cfg1_decode")
    ref = port.decode(layer, X)[0]
    got = dm.granite_moe(layer, X[0])
    err = rel_l2(got, ref)
    assert err <= REL_L2_TOL, err
    # the fp32 CUDA-core path tracks the reference to fp32 rounding
    assert err < 1e-5, err


def test_bailing_moe_groups(dlib, port):
    layer = synth.make_layer(hidden=2048, n_exp=64, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                             n_group_used=4, w_scale=2.5, bias=True, seed=31)
    X = synth.make_tokens(layer, 3, 31)
    ref = port.decode(layer, X)
    for t in range(3):
        got = dm.bailing_moe(layer, X[t])
        assert rel_l2(got, ref[t]) <= REL_L2_TOL


def test_moe_op_with_shared(dlib, port):
    layer = synth.make_layer(hidden=2048, n_exp=32, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                             n_group_used=4, w_scale=2.5, bias=True, shared_inter=512, seed=32)
    X = synth.make_tokens(layer, 1, 32)
    ref = port.decode(layer, X)
    port.shared_add(layer, X, ref)
    ep, ec = layer.ptr_table()
    gi = np.ascontiguousarray(layer.gate_inp)
    p = dm.M6MoeP()
    p.exp_ptrs = ep.ctypes.data_as(dm._u64)
    p.exp_codes = ec.ctypes.data_as(dm._i)
    p.gate_inp = gi.ctypes.data_as(dm._f)
    p.probs_b = layer.probs_b.ctypes.data_as(dm._f)
    p.n_exp, p.n_used, p.n_group, p.n_group_used, p.norm_w = 32, 8, 8, 4, 1
    p.w_scale = 2.5
    p.inter, p.n_in, p.n_out = 512, 2048, 2048
    p.sh_g, p.sh_u, p.sh_d = layer.sh_gate.ctypes.data, layer.sh_up.ctypes.data, layer.sh_down.ctypes.data
    p.csg, p.csu, p.csd, p.sh_ff = 5, 5, 4, 512
    out = np.empty(2048, np.float32)
    dm.lib().m6_moe_op(X[0].ctypes.data_as(dm._f), ct.byref(p), out.ctypes.data_as(dm._f))
    assert rel_l2(out, ref[0]) <= REL_L2_TOL


def test_granite_shexp(dlib, port):
    rng = np.random.default_rng(33)
    h, shi = 2048, 512
    g = synth.quant_matrix(rng, 5, 1, shi, h)[0]
    u = synth.quant_matrix(rng, 5, 1, shi, h)[0]
    d = synth.quant_matrix(rng, 4, 1, h, shi)[0]
    gw = (rng.standard_normal(h).astype(np.float32) * 0.05).astype(np.float32)
    x = synth.rms_normed(rng, 1, h)[0]
    shp = np.array([g.ctypes.data, u.ctypes.data, d.ctypes.data, gw.ctypes.data], np.uint64)
    shc = np.array([5, 5, 4, 9], np.int32)
    ref = np.empty(h, np.float32)
    port.L.orc_granite_shexp(x.ctypes.data_as(dm._f), shp.ctypes.data_as(dm._u64), shc.ctypes.data_as(dm._i),
                             shi, h, ref.ctypes.data_as(dm._f))
    out = np.empty(h, np.float32)
    sg = np.zeros(1, np.float32)
    shg = np.zeros(h, np.float32)
    dm.lib().m6_granite_shexp(x.ctypes.data_as(dm._f), shp.ctypes.data_as(dm._u64), shc.ctypes.data_as(dm._i),
                              sg.ctypes.data_as(dm._f), None, shg.ctypes.data_as(dm._f), out.ctypes.data_as(dm._f),
                              shi, h)
    assert rel_l2(out, ref) <= REL_L2_TOL
    assert abs(sg[0] - float(np.dot(gw.astype(np.float64), x))) < 1e-3


# ----------------------------------------------------------------------------- prefill
def test_moe_tok_cfg2_shape(dlib, port):
    layer, X = synth.make_config("cfg2_prefill", tokens=64)
    order, wtop = port.route(layer, X)
    ref = port.moe_tok(layer, X, order, wtop)
    got = dm.moe_tok(layer, X, order, wtop)
    assert rel_l2(got, ref) <= REL_L2_TOL


@pytest.mark.parametrize("T", [12, 200])   # 200 x 4 assignments: the tensor-core path
def test_moe_tok_skips_invalid_and_zero_tokens(dlib, port, T):
    layer = synth.make_layer(hidden=512, n_exp=16, n_used=4, inter=256, seed=41)
    X = synth.make_tokens(layer, T, 41)
    order, wtop = port.route(layer, X)
    order[0, 1] = -1          # skipped by the reference's scatter (src/m6_moe_tok.c:154)
    order[3, 2] = 16          # out of range: skipped as well
    if T > 12:
        rng = np.random.default_rng(3)
        order[rng.random(order.shape) < 0.2] = -1
        order[rng.random(order.shape) < 0.1] = 99
    ref = port.moe_tok(layer, X, order, wtop)
    got = dm.moe_tok(layer, X, order, wtop)
    assert rel_l2(got, ref) <= REL_L2_TOL
    # T == 0 is a no-op
    empty = dm.moe_tok(layer, X[:0], order[:0], wtop[:0])
    assert empty.shape == (0, 512)


def test_forward_layer_with_shared(dlib, port):
    layer = synth.make_layer(hidden=2048, n_exp=64, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                             n_group_used=4, w_scale=2.5, shared_inter=512, bias=True, seed=42)
    X = synth.make_tokens(layer, 40, 42)
    ref = port.layer_forward(layer, X)
    order = np.empty((40, 8), np.int32)
    wtop = np.empty((40, 8), np.float32)
    got = np.empty((40, 2048), np.float32)
    keep = []
    d = dm.layer_desc(layer, keep)
    rc = dm.lib().draco_b200_moe_forward(ct.byref(d), X.ctypes.data, 40, got.ctypes.data, order.ctypes.data,
                                         wtop.ctypes.data, None)
    assert rc == 0, dm.last_error()
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(order, o_ref)
    assert np.array_equal(bits(wtop), bits(w_ref))
    assert rel_l2(got, ref) <= REL_L2_TOL


# ----------------------------------------------------------------------------- kernels
@pytest.mark.parametrize("code,n_out,n_in", [(5, 96, 2048), (4, 128, 768), (0, 64, 512), (0, 32, 96)])
def test_gemv_and_dequant(dlib, port, code, n_out, n_in):
    rng = np.random.default_rng(code * 7 + n_in)
    W = synth.quant_matrix(rng, code, 1, n_out, n_in)[0]
    x = rng.standard_normal(n_in).astype(np.float32)
    ref = port.gemv(code, x, W, n_out, n_in)
    y = np.zeros(n_out, np.float32)
    assert dm.lib().m5_gemv(code, x.ctypes.data_as(dm._f), W.ctypes.data_as(dm._u8), n_out, n_in,
                            y.ctypes.data_as(dm._f)) == 0
    assert rel_l2(y, ref) < 1e-5
    # range entry writes only [o0, o1)
    y2 = np.full(n_out, 7.0, np.float32)
    assert dm.lib().m5_gemv_range(code, x.ctypes.data_as(dm._f), W.ctypes.data_as(dm._u8), n_out, n_in,
                                  y2.ctypes.data_as(dm._f), 8, 24) == 0
    assert np.all(y2[:8] == 7.0) and np.all(y2[24:] == 7.0)
    assert rel_l2(y2[8:24], ref[8:24]) < 1e-5
    deq = port.dequant(code, W, n_out, n_in)
    row = np.empty(n_in, np.float32)
    rb = synth.row_bytes(code, n_in)
    assert dm.lib().m5_dequant_row(code, W[5 * rb:].ctypes.data_as(dm._u8), n_in, row.ctypes.data_as(dm._f)) == 0
    assert np.allclose(row, deq[5], rtol=2e-7, atol=1e-9)


def test_gemm_dense(dlib, port):
    rng = np.random.default_rng(51)
    n_out, n_in, T = 192, 1024, 37
    W = synth.quant_matrix(rng, 5, 1, n_out, n_in)[0]
    X = rng.standard_normal((T, n_in)).astype(np.float32)
    ref = np.stack([port.gemv(5, X[t], W, n_out, n_in) for t in range(T)])
    Y = np.zeros((T, n_out), np.float32)
    assert dm.lib().m5_gemm_auto(5, X.ctypes.data, W.ctypes.data, T, n_out, n_in, Y.ctypes.data) == 0
    assert rel_l2(Y, ref) < 1e-5
    assert dm.lib().m5_gemm_auto(2, X.ctypes.data, W.ctypes.data, T, n_out, n_in, Y.ctypes.data) == -1


@pytest.mark.parametrize("code", [5, 4])
def test_gemvn_matches_reference(dlib, port, code):
    rng = np.random.default_rng(60 + code)
    E, n_out, n_in, N = 12, 256, 1024, 5
    W = synth.quant_matrix(rng, code, E, n_out, n_in)
    per = W.shape[1]
    idx = np.array([7, 2, 11, 2, 0], np.int32)
    for x_stride in (0, n_in):
        x = rng.standard_normal(N * n_in).astype(np.float32)
        ref = np.concatenate([port.gemv(code, x[e * x_stride:e * x_stride + n_in], W[idx[e]], n_out, n_in)
                              for e in range(N)])
        y = np.zeros(N * n_out, np.float32)
        fn = dm.lib().m5_gemvn_q4k if code == 5 else dm.lib().m5_gemvn_q6k
        assert fn(x.ctypes.data_as(dm._f), x_stride, W.ctypes.data_as(dm._u8), idx.ctypes.data_as(dm._i), per,
                  n_out, n_in, N, y.ctypes.data_as(dm._f)) == 0
        assert rel_l2(y, ref) < 1e-5


# ----------------------------------------------------------------------------- Q8_K
def test_q8k_quantize_and_dots_bitexact(dlib, port):
    rng = np.random.default_rng(71)
    n_in, rows = 2048, 64
    x = synth.rms_normed(rng, 1, n_in)[0]
    x[256:512] = 0.0                     # an all-zero block: d = 0
    d_ref, q_ref, bs_ref = port.q8k_quantize(x)
    d = np.zeros(n_in // 256, np.float32)
    q = np.zeros(n_in, np.int8)
    bs = np.zeros(n_in // 16, np.int16)
    L = dm.lib()
    assert L.draco_b200_q8k_quantize(x.ctypes.data_as(dm._f), n_in, d.ctypes.data_as(dm._f),
                                     q.ctypes.data_as(dm._i8), bs.ctypes.data_as(dm._i16)) == 0
    assert np.array_equal(q, q_ref) and np.array_equal(bs, bs_ref) and np.array_equal(bits(d), bits(d_ref))
    for code in (5, 4):
        W = synth.quant_matrix(rng, code, 1, rows, n_in)[0]
        nb = n_in // 256
        out2 = np.zeros(rows * nb * 2, np.int32)
        assert L.draco_b200_q8k_block_dots(code, W.ctypes.data_as(dm._u8), rows, n_in, q.ctypes.data_as(dm._i8),
                                           bs.ctypes.data_as(dm._i16), out2.ctypes.data_as(dm._i32)) == 0
        rb = synth.row_bytes(code, n_in)
        bb = 144 if code == 5 else 210
        for r in range(rows):
            for b in range(nb):
                blk = W[r * rb + b * bb:].ctypes.data_as(dm._u8)
                a = np.zeros(1, np.int32)
                m = np.zeros(1, np.int32)
                if code == 5:
                    port.L.orc_q4k_q8k_block(blk, q[b * 256:].ctypes.data_as(dm._i8),
                                             bs[b * 16:].ctypes.data_as(dm._i16), a.ctypes.data_as(dm._i32),
                                             m.ctypes.data_as(dm._i32))
                else:
                    port.L.orc_q6k_q8k_block(blk, q[b * 256:].ctypes.data_as(dm._i8), a.ctypes.data_as(dm._i32))
                assert out2[(r * nb + b) * 2] == a[0] and out2[(r * nb + b) * 2 + 1] == m[0], (code, r, b)
        y = np.zeros(rows, np.float32)
        assert L.draco_b200_gemv_q8k(code, W.ctypes.data_as(dm._u8), rows, n_in, q.ctypes.data_as(dm._i8),
                                     d.ctypes.data_as(dm._f), bs.ctypes.data_as(dm._i16), y.ctypes.data_as(dm._f)) == 0
        y_ref = port.gemv_q8k(code, d, q, bs, W, rows, n_in)
        assert np.array_equal(bits(y), bits(y_ref))


# ----------------------------------------------------------------------------- tensor-core path
@pytest.fixture
def gemm_path(dlib):
    old = dlib.draco_b200_set_gemm_path(0)
    yield dlib.draco_b200_set_gemm_path
    dlib.draco_b200_set_gemm_path(old)


@pytest.mark.parametrize("code_gu,code_d,T", [(5, 4, 64), (4, 5, 48), (5, 4, 3), (5, 5, 200)])
def test_tensor_core_moe_tok(dlib, port, gemm_path, code_gu, code_d, T):
    """tcgen05 grouped GEMM (fp16 operands, fp32 accumulation) vs the fp32 oracle."""
    layer = synth.make_layer(hidden=2048, n_exp=16, n_used=8, inter=768, seed=80 + code_gu + T,
                             code_gu=code_gu, code_d=code_d)
    X = synth.make_tokens(layer, T, 80 + T)
    order, wtop = port.route(layer, X)
    ref = port.moe_tok(layer, X, order, wtop)
    gemm_path(2)
    got = dm.moe_tok(layer, X, order, wtop)
    err = rel_l2(got, ref)
    assert err <= REL_L2_TOL, err
    gemm_path(1)
    simt = dm.moe_tok(layer, X, order, wtop)
    assert rel_l2(simt, ref) < 1e-5


@pytest.mark.parametrize("n_exp,T", [(8, 300), (64, 300), (256, 300)])
def test_tensor_core_hot_expert_many_tiles(dlib, port, gemm_path, n_exp, T):
    """One expert receives every token and one other half of them: several token tiles
    (128-token tiles with 8 experts, 64-token tiles with 64 and 256: the tile height follows the
    average load per expert)."""
    layer = synth.make_layer(hidden=1024, n_exp=n_exp, n_used=2, inter=512, seed=90)
    X = synth.make_tokens(layer, T, 90)
    order = np.zeros((T, 2), np.int32)
    order[:, 0] = 3
    order[:, 1] = np.where(np.arange(T) % 2 == 0, 5, 3)
    wtop = np.full((T, 2), 0.5, np.float32)
    ref = port.moe_tok(layer, X, order, wtop)
    gemm_path(2)
    got = dm.moe_tok(layer, X, order, wtop)
    assert rel_l2(got, ref) <= REL_L2_TOL


def test_tensor_core_layer_k2_shape(dlib, port, gemm_path):
    """K2 expert shape (H 7168, F 2048) with sigmoid routing, bias, scale and a shared expert."""
    layer = synth.make_layer(hidden=7168, n_exp=16, n_used=8, inter=2048, scoring="sigmoid", w_scale=2.827,
                             bias=True, shared_inter=2048, seed=91)
    X = synth.make_tokens(layer, 40, 91)
    ref = port.layer_forward(layer, X)
    gemm_path(2)
    got = dm.forward(layer, X)
    assert rel_l2(got, ref) <= REL_L2_TOL
