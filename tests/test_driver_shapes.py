"""The reference's numpy/ctypes model drivers, restated call for call, bound once to this
library and once to the reference's own C (oracle/_ref), on the same synthetic GGUF-layout
tensors.  Only the shared-object paths differ between the two runs, which is the drop-in
contract: a driver pointed at this library (M6_SO, the m6_moe_tok.so / m5 names) must get the
reference's results.

  qwen35 decode FFN     src/qwen35_engine.py:293-308  (m6_granite_moe + m6_granite_shexp,
                        then out = mo + out), argtypes of :118-125
  qwen35 chunk prefill  src/qwen35_prefill.py:170-207 (numpy softmax routing, m6_moe_tok with
                        the injected DQ/GA pointers, the shared expert through the fused GEMMs
                        m5_gemm_q4k/q6k and a scalar sigmoid gate), argtypes of :65-83
  K2 decode MoE         src/k2_engine.py:498-562, the K2_BATCH branch (numpy sigmoid routing,
                        m5_gemvn_q4k for gate and up with x_stride 0, m5_gemvn_q6k for down with
                        x_stride MOE_INTER, weighted sum in numpy), argtypes of :100-106

Bar: rel-L2 <= 1e-3 between the two runs (the layer bar of the parity tests).
"""
import ctypes as ct
import os

import numpy as np
import pytest

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3
pf = lambda a: a.ctypes.data_as(ct.POINTER(ct.c_float))   # noqa: E731  (the drivers' helper)
p8 = lambda a: a.ctypes.data_as(ct.POINTER(ct.c_uint8))   # noqa: E731


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def libs_for(which):
    """{m6_engine, m6_moe_tok, m5_gemm, m5_gemm_fused, m5_batch8_k}: this library under every
    name, or the reference's objects."""
    from oracle.oracle import REF_DIR, ref_available
    if which == "draco":
        L = ct.CDLL(dm.LIB_PATH)
        return {k: L for k in ("m6_engine", "m6_moe_tok", "m5_gemm", "m5_gemm_fused", "m5_batch8_k")}
    if not ref_available():
        pytest.skip("oracle/_ref not built")
    j = lambda n: ct.CDLL(os.path.join(REF_DIR, n))   # noqa: E731
    out = {"m6_engine": j("m6_engine.so"), "m6_moe_tok": j("m6_moe_tok.so"), "m5_gemm": j("m5_gemm.so"),
           "m5_gemm_fused": j("m5_gemm_fused.so"), "m5_batch8_k": j("m5_batch8_k.so")}
    out["m6_engine"].m6_init_dl.argtypes = [ct.c_char_p] * 5
    assert out["m6_engine"].m6_init_dl(*[os.path.join(REF_DIR, "m5_kern_scalar.so").encode()] * 5) == 0
    return out


def qwen35_layer(seed):
    layer = synth.make_layer(hidden=2048, n_exp=64, n_used=8, inter=512, shared_inter=1024, seed=seed)
    rng = np.random.default_rng(seed + 1)
    gi_sh = (rng.standard_normal(2048) * 0.05).astype(np.float32)   # ffn_gate_inp_shexp (F32)
    return layer, gi_sh


# --------------------------------------------------------------------------- qwen35 decode
def qwen35_ffn(libs, layer, gi_sh, xn):
    """src/qwen35_engine.py:293-308 with the argtypes of :118-125."""
    M6E = libs["m6_engine"]
    M6E.m6_granite_shexp.argtypes = [ct.POINTER(ct.c_float), ct.POINTER(ct.c_uint64), ct.POINTER(ct.c_int),
                                     ct.POINTER(ct.c_float), ct.POINTER(ct.c_float), ct.POINTER(ct.c_float),
                                     ct.POINTER(ct.c_float), ct.c_int, ct.c_int]
    M6E.m6_granite_shexp.restype = None
    M6E.m6_granite_moe.argtypes = [ct.POINTER(ct.c_float), ct.POINTER(ct.c_uint64), ct.POINTER(ct.c_int),
                                   ct.POINTER(ct.c_float), ct.c_int, ct.c_int, ct.c_int, ct.c_int, ct.c_int,
                                   ct.POINTER(ct.c_float), ct.POINTER(ct.c_float)]
    M6E.m6_granite_moe.restype = None
    H, N_EXP, N_USED, EXP_FFN, SHEXP_FFN = layer.hidden, layer.n_exp, layer.n_used, layer.inter, layer.shared_inter
    ep, ec = layer.ptr_table()
    gi = np.ascontiguousarray(layer.gate_inp)
    shp = np.array([layer.sh_gate.ctypes.data, layer.sh_up.ctypes.data, layer.sh_down.ctypes.data,
                    gi_sh.ctypes.data], np.uint64)
    shc = np.array([layer.code_gu, layer.code_gu, layer.code_d, 9], np.int32)
    M = dict(ep=ep.ctypes.data_as(ct.POINTER(ct.c_uint64)), ec=ec.ctypes.data_as(ct.POINTER(ct.c_int)), gi=pf(gi),
             shp=shp.ctypes.data_as(ct.POINTER(ct.c_uint64)), shc=shc.ctypes.data_as(ct.POINTER(ct.c_int)),
             scratch=np.zeros(3 * N_USED * EXP_FFN + N_USED * H, np.float32), sg=np.zeros(1, np.float32),
             mo=np.zeros(H, np.float32), sh=np.zeros(2 * SHEXP_FFN, np.float32), shg=np.zeros(H, np.float32))
    out = np.zeros(H, np.float32)
    M6E.m6_granite_moe(pf(xn), M["ep"], M["ec"], M["gi"], N_EXP, N_USED, EXP_FFN, H, H, pf(M["scratch"]),
                       pf(M["mo"]))
    M6E.m6_granite_shexp(pf(xn), M["shp"], M["shc"], pf(M["sg"]), pf(M["sh"]), pf(M["shg"]), pf(out), SHEXP_FFN, H)
    out[:] = M["mo"] + out
    return out, M["sg"][0]


def test_qwen35_decode_ffn(dlib):
    layer, gi_sh = qwen35_layer(81)
    X = synth.make_tokens(layer, 3, 82)
    for t in range(3):
        a, sga = qwen35_ffn(libs_for("draco"), layer, gi_sh, X[t])
        b, sgb = qwen35_ffn(libs_for("reference"), layer, gi_sh, X[t])
        assert rel_l2(a, b) <= REL_L2_TOL, (t, rel_l2(a, b))
        assert abs(sga - sgb) <= 1e-4 * max(1.0, abs(sgb))


# --------------------------------------------------------------------------- qwen35 prefill
def qwen35_ffn_chunk(libs, layer, gi_sh, X2n):
    """src/qwen35_prefill.py:170-207 (routing in numpy, the experts in m6_moe_tok, the shared expert
    through the fused GEMMs), the bindings of :65-83."""
    G, MT, FG = libs["m5_gemm"], libs["m6_moe_tok"], libs["m5_gemm_fused"]
    MT.m6_moe_tok.restype = None
    MT.m6_moe_tok.argtypes = [ct.c_void_p] * 8 + [ct.c_int] * 6 + [ct.c_void_p] * 3
    dq_fp = ct.cast(G.m5_dequant_row, ct.c_void_p)
    FG.m5_gemm_auto.restype = ct.c_int
    FG.m5_gemm_auto.argtypes = [ct.c_int] + [ct.c_void_p] * 2 + [ct.c_int] * 3 + [ct.c_void_p]
    fused_fp = ct.cast(FG.m5_gemm_auto, ct.c_void_p)
    fused_fn = {4: FG.m5_gemm_q6k, 5: FG.m5_gemm_q4k}
    for fn in fused_fn.values():
        fn.restype = None
        fn.argtypes = [ct.POINTER(ct.c_float), ct.POINTER(ct.c_uint8), ct.c_int, ct.c_int, ct.c_int,
                       ct.POINTER(ct.c_float)]
    nth = os.cpu_count() or 8
    wbuf = np.zeros(nth * 8208, np.float32)

    def gemm(code, X, w_ptr, n_out, n_in):
        T = X.shape[0]
        Y = np.empty((T, n_out), np.float32)
        fused_fn[code](X.ctypes.data_as(ct.POINTER(ct.c_float)), ct.cast(w_ptr, ct.POINTER(ct.c_uint8)), T, n_out,
                       n_in, pf(Y))
        return Y

    T, H = X2n.shape
    FF, NEXP, NUSED = layer.inter, layer.n_exp, layer.n_used
    gi = layer.gate_inp
    lg = X2n @ gi.T
    lg -= lg.max(1, keepdims=True)
    P = np.exp(lg)
    P /= P.sum(1, keepdims=True)
    order = np.argsort(-P, axis=1, kind="stable")[:, :NUSED]
    wtop = np.take_along_axis(P, order, 1)
    wtop /= np.maximum(wtop.sum(1, keepdims=True), 6.103515625e-5)
    out = np.zeros((T, H), np.float32)
    order_c = np.ascontiguousarray(order, np.int32)
    wtop_c = np.ascontiguousarray(wtop, np.float32)
    work = np.empty(T * NUSED * (H + 3 * FF + H), np.float32)
    iwork = np.empty(T * NUSED * 2 + NEXP + 1, np.int32)
    ep, ec = layer.ptr_table()
    MT.m6_moe_tok(dq_fp, fused_fp, wbuf.ctypes.data, pf(X2n), pf(order_c), pf(wtop_c),
                  ep.ctypes.data_as(ct.POINTER(ct.c_uint64)), ec.ctypes.data_as(ct.POINTER(ct.c_int)),
                  T, NUSED, FF, H, H, NEXP, pf(out), pf(work), pf(iwork))
    gsc = 1.0 / (1.0 + np.exp(-(X2n @ gi_sh)))
    shg = gemm(layer.code_gu, X2n, layer.sh_gate.ctypes.data, layer.shared_inter, H)
    shu = gemm(layer.code_gu, X2n, layer.sh_up.ctypes.data, layer.shared_inter, H)
    act = np.ascontiguousarray(shg / (1.0 + np.exp(-shg)) * shu)
    shd = gemm(layer.code_d, act, layer.sh_down.ctypes.data, H, layer.shared_inter)
    return out + shd * gsc[:, None]


@pytest.mark.parametrize("T", [5, 96])
def test_qwen35_prefill_ffn_chunk(dlib, T):
    layer, gi_sh = qwen35_layer(83)
    X = np.ascontiguousarray(synth.make_tokens(layer, T, 84))
    a = qwen35_ffn_chunk(libs_for("draco"), layer, gi_sh, X)
    b = qwen35_ffn_chunk(libs_for("reference"), layer, gi_sh, X)
    assert rel_l2(a, b) <= REL_L2_TOL, rel_l2(a, b)


# --------------------------------------------------------------------------- K2 decode
def k2_moe_ffn(libs, layer, h2, R_SCALING):
    """src/k2_engine.py:498-562, K2_BATCH branch, with the argtypes of :100-106; the shared expert
    of the driver (:577-591) is left out here (the same GEMVs)."""
    LIB_B = libs["m5_batch8_k"]
    for fn in ("m5_gemvn_q4k", "m5_gemvn_q6k"):
        f = getattr(LIB_B, fn)
        f.restype = ct.c_int
        f.argtypes = [ct.POINTER(ct.c_float), ct.c_long, ct.POINTER(ct.c_uint8), ct.POINTER(ct.c_int), ct.c_long,
                      ct.c_int, ct.c_int, ct.c_int, ct.POINTER(ct.c_float)]
    H, NUSED, MOE_INTER = layer.hidden, layer.n_used, layer.inter
    logits = layer.gate_inp @ h2
    sc = 1.0 / (1.0 + np.exp(-np.asarray(logits, np.float32)))
    sel = np.argsort(-(sc + layer.probs_b), kind="stable")[:NUSED]
    rw = sc[sel]
    rw = rw / rw.sum() * R_SCALING
    sel_a = np.ascontiguousarray(sel, np.int32)
    pi_ = ct.POINTER(ct.c_int)
    G = np.empty(NUSED * MOE_INTER, np.float32)
    U = np.empty(NUSED * MOE_INTER, np.float32)
    ex_per, ux_per, dx_per = layer.gate.shape[1], layer.up.shape[1], layer.down.shape[1]
    rc = LIB_B.m5_gemvn_q4k(pf(h2), 0, p8(layer.gate), sel_a.ctypes.data_as(pi_), ex_per, MOE_INTER, H, NUSED, pf(G))
    rc += LIB_B.m5_gemvn_q4k(pf(h2), 0, p8(layer.up), sel_a.ctypes.data_as(pi_), ux_per, MOE_INTER, H, NUSED, pf(U))
    assert rc == 0, f"batch q4k rc={rc}"
    gu = (G / (1.0 + np.exp(-G)) * U).reshape(NUSED, MOE_INTER).astype(np.float32)
    D = np.empty(NUSED * H, np.float32)
    rc = LIB_B.m5_gemvn_q6k(pf(np.ascontiguousarray(gu.ravel())), MOE_INTER, p8(layer.down),
                            sel_a.ctypes.data_as(pi_), dx_per, H, MOE_INTER, NUSED, pf(D))
    assert rc == 0, f"batch q6k rc={rc}"
    return (D.reshape(NUSED, H) * rw[:, None]).sum(0)


def test_k2_decode_moe_ffn(dlib):
    layer = synth.make_layer(hidden=7168, n_exp=48, n_used=8, inter=2048, scoring="sigmoid", w_scale=2.827,
                             bias=True, seed=85)
    X = synth.make_tokens(layer, 1, 86)
    for t in range(1):
        a = k2_moe_ffn(libs_for("draco"), layer, X[t], 2.827)
        b = k2_moe_ffn(libs_for("reference"), layer, X[t], 2.827)
        assert rel_l2(a, b) <= REL_L2_TOL, (t, rel_l2(a, b))
