"""ctypes bindings for the CPU checkers of the MoE hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference arm.  The product (dracomancer_llmengine_b200) never imports this module.

Two checkers:
  * `Port`  -- oracle/libmoe_oracle.so, this repository's C restatement of the reference's
    algorithm (moe_oracle.c), always buildable from source here or on the GPU box;
  * `Ref`   -- oracle/_ref/*.so, the reference's own C compiled unmodified by
    `make -C oracle ref` from the reference sources (only where they are present; the
    built .so files travel with the repository snapshot).
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
PORT_SO = os.path.join(HERE, "libmoe_oracle.so")

_f = ct.POINTER(ct.c_float)
_i = ct.POINTER(ct.c_int)
_u64 = ct.POINTER(ct.c_uint64)
_u8 = ct.POINTER(ct.c_uint8)
_i8 = ct.POINTER(ct.c_int8)
_i16 = ct.POINTER(ct.c_int16)
_i32 = ct.POINTER(ct.c_int32)


def pf(a):
    return a.ctypes.data_as(_f)


def pi(a):
    return a.ctypes.data_as(_i)


def pu64(a):
    return a.ctypes.data_as(_u64)


def build_port() -> str:
    if not os.path.exists(PORT_SO) or os.path.getmtime(PORT_SO) < max(
            os.path.getmtime(os.path.join(HERE, f)) for f in ("moe_oracle.c", "moe_oracle.h")):
        subprocess.run(["make", "-s", "-C", HERE, "libmoe_oracle.so"], check=True)
    return PORT_SO


def ref_available() -> bool:
    return all(os.path.exists(os.path.join(REF_DIR, n)) for n in
               ("m5_kern_scalar.so", "m6_engine.so", "m6_moe_tok.so", "m5_gemm.so",
                "m5_gemm_fused.so", "m5_batch8_k.so"))


class Port:
    """The C restatement (moe_oracle.c)."""

    def __init__(self):
        L = ct.CDLL(build_port())
        self.L = L
        L.orc_gemv_range.argtypes = [ct.c_int, _f, _u8, ct.c_int, ct.c_int, _f, ct.c_int, ct.c_int]
        L.orc_gemv_range.restype = ct.c_int
        L.orc_dequant_row.argtypes = [ct.c_int, _u8, ct.c_int, _f]
        L.orc_dequant_row.restype = ct.c_int
        L.orc_route_softmax.argtypes = [_f, _f, ct.c_int, ct.c_int, ct.c_int, _i, _f, _f]
        L.orc_route_softmax.restype = None
        L.orc_route_sigmoid.argtypes = [_f, _f, _f, ct.c_int, ct.c_int, ct.c_int, ct.c_int,
                                        ct.c_int, ct.c_float, ct.c_int, _i, _f, _f]
        L.orc_route_sigmoid.restype = None
        L.orc_route_batch.argtypes = [ct.c_int, _f, ct.c_int, _f, _f] + [ct.c_int] * 5 + [ct.c_float, ct.c_int, _i, _f]
        L.orc_route_batch.restype = None
        L.orc_granite_moe.argtypes = [_f, _u64, _i, _f] + [ct.c_int] * 5 + [_f]
        L.orc_granite_moe.restype = None
        L.orc_bailing_moe.argtypes = [_f, _u64, _i, _f, _f] + [ct.c_int] * 5 + [ct.c_float] + [ct.c_int] * 3 + [_f]
        L.orc_bailing_moe.restype = None
        L.orc_granite_shexp.argtypes = [_f, _u64, _i, ct.c_int, ct.c_int, _f]
        L.orc_granite_shexp.restype = None
        L.orc_shared_add.argtypes = [_f, _u8, _u8, _u8] + [ct.c_int] * 6 + [_f]
        L.orc_shared_add.restype = None
        L.orc_shared_add_batch.argtypes = [_f, ct.c_int, _u8, _u8, _u8] + [ct.c_int] * 6 + [_f]
        L.orc_shared_add_batch.restype = None
        L.orc_moe_tok.argtypes = [_f, _i, _f, _u64, _i] + [ct.c_int] * 6 + [_f]
        L.orc_moe_tok.restype = None
        L.orc_q8k_quantize.argtypes = [_f, ct.c_int, _f, _i8, _i16]
        L.orc_q8k_quantize.restype = None
        L.orc_q4k_q8k_block.argtypes = [_u8, _i8, _i16, _i32, _i32]
        L.orc_q4k_q8k_block.restype = None
        L.orc_q6k_q8k_block.argtypes = [_u8, _i8, _i32]
        L.orc_q6k_q8k_block.restype = None
        L.orc_gemv_q8k.argtypes = [ct.c_int, _f, _i8, _i16, _u8, ct.c_int, ct.c_int, _f]
        L.orc_gemv_q8k.restype = None
        L.orc_expf_array.argtypes = [_f, _f, ct.c_long]
        L.orc_expf_array.restype = None

    # -- kernels --
    def gemv(self, code, x, W, n_out, n_in):
        y = np.zeros(n_out, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.L.orc_gemv_range(code, pf(x), W.ctypes.data_as(_u8), n_out, n_in, pf(y), 0, n_out)
        assert rc == 0
        return y

    def dequant(self, code, W, n_out, n_in):
        from dracomancer_llmengine_b200.synth import row_bytes
        rb = row_bytes(code, n_in)
        flat = np.ascontiguousarray(W).reshape(-1)
        out = np.empty((n_out, n_in), np.float32)
        for r in range(n_out):
            self.L.orc_dequant_row(code, flat[r * rb:(r + 1) * rb].ctypes.data_as(_u8), n_in, pf(out[r]))
        return out

    # -- routers --
    def route(self, layer, x):
        """(idx int32[T, K], w fp32[T, K]) for every token row of x, C-router semantics (one
        OpenMP thread per token)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = x.shape[0]
        idx = np.zeros((T, layer.n_used), np.int32)
        w = np.zeros((T, layer.n_used), np.float32)
        gi = np.ascontiguousarray(layer.gate_inp, np.float32)
        sig = layer.scoring != "softmax"
        pb = pf(layer.probs_b) if sig and layer.probs_b is not None else None
        self.L.orc_route_batch(1 if sig else 0, pf(x), T, pf(gi), pb, layer.n_exp, layer.n_used,
                               layer.n_group if sig else 1, layer.n_group_used, layer.norm_w,
                               ct.c_float(layer.w_scale if sig else 0.0), layer.hidden, pi(idx), pf(w))
        return idx, w

    def route_probs(self, layer, x):
        """(idx, w, probs fp32[T, E]) with the per-token C router (probs: the softmax or sigmoid
        scores before selection)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = x.shape[0]
        idx = np.zeros((T, layer.n_used), np.int32)
        w = np.zeros((T, layer.n_used), np.float32)
        P = np.zeros((T, layer.n_exp), np.float32)
        gi = np.ascontiguousarray(layer.gate_inp, np.float32)
        pb = pf(layer.probs_b) if layer.probs_b is not None else None
        for t in range(T):
            if layer.scoring == "softmax":
                self.L.orc_route_softmax(pf(x[t]), pf(gi), layer.n_exp, layer.n_used, layer.hidden,
                                         pi(idx[t]), pf(w[t]), pf(P[t]))
            else:
                self.L.orc_route_sigmoid(pf(x[t]), pf(gi), pb, layer.n_exp, layer.n_used, layer.n_group,
                                         layer.n_group_used, layer.norm_w, ct.c_float(layer.w_scale), layer.hidden,
                                         pi(idx[t]), pf(w[t]), pf(P[t]))
        return idx, w, P

    # -- layers --
    def decode(self, layer, x):
        """Routed experts for each token row independently (decode semantics, no shared expert)."""
        ep, ec = layer.ptr_table()
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        out = np.zeros((x.shape[0], layer.hidden), np.float32)
        gi = np.ascontiguousarray(layer.gate_inp, np.float32)
        for t in range(x.shape[0]):
            if layer.scoring == "softmax":
                self.L.orc_granite_moe(pf(x[t]), pu64(ep), pi(ec), pf(gi), layer.n_exp, layer.n_used,
                                       layer.inter, layer.hidden, layer.hidden, pf(out[t]))
            else:
                pb = pf(layer.probs_b) if layer.probs_b is not None else None
                self.L.orc_bailing_moe(pf(x[t]), pu64(ep), pi(ec), pf(gi), pb, layer.n_exp,
                                       layer.n_used, layer.n_group, layer.n_group_used, layer.norm_w,
                                       ct.c_float(layer.w_scale), layer.inter, layer.hidden,
                                       layer.hidden, pf(out[t]))
        return out

    def shared_add(self, layer, x, out):
        """out[t] += ungated shared expert(x[t]) for every row (one OpenMP thread per row)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        assert out.flags.c_contiguous and out.dtype == np.float32
        self.L.orc_shared_add_batch(pf(x), x.shape[0], layer.sh_gate.ctypes.data_as(_u8),
                                    layer.sh_up.ctypes.data_as(_u8), layer.sh_down.ctypes.data_as(_u8),
                                    layer.code_gu, layer.code_gu, layer.code_d, layer.shared_inter,
                                    layer.hidden, layer.hidden, pf(out))
        return out

    def moe_tok(self, layer, X, order, wtop):
        ep, ec = layer.ptr_table()
        X = np.ascontiguousarray(X, np.float32)
        order = np.ascontiguousarray(order, np.int32)
        wtop = np.ascontiguousarray(wtop, np.float32)
        out = np.zeros((X.shape[0], layer.hidden), np.float32)
        self.L.orc_moe_tok(pf(X), pi(order), pf(wtop), pu64(ep), pi(ec), X.shape[0], layer.n_used,
                           layer.inter, layer.hidden, layer.hidden, layer.n_exp, pf(out))
        return out

    def layer_forward(self, layer, X, order=None, wtop=None):
        """Whole layer on a token batch: C-router semantics routing, routed experts (prefill
        order), ungated shared expert when the layer has one."""
        if order is None:
            order, wtop = self.route(layer, X)
        out = self.moe_tok(layer, X, order, wtop)
        if layer.shared_inter:
            self.shared_add(layer, X, out)
        return out

    def expf(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.orc_expf_array(pf(x), pf(y), x.size)
        return y

    # -- Q8_K --
    def q8k_quantize(self, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        nb = x.size // 256
        d = np.zeros(nb, np.float32)
        q = np.zeros(nb * 256, np.int8)
        bs = np.zeros(nb * 16, np.int16)
        self.L.orc_q8k_quantize(pf(x), x.size, pf(d), q.ctypes.data_as(_i8), bs.ctypes.data_as(_i16))
        return d, q, bs

    def gemv_q8k(self, code, d, q, bs, W, n_out, n_in):
        y = np.zeros(n_out, np.float32)
        self.L.orc_gemv_q8k(code, pf(d), q.ctypes.data_as(_i8), bs.ctypes.data_as(_i16),
                            W.ctypes.data_as(_u8), n_out, n_in, pf(y))
        return y


class Ref:
    """The reference's own C (oracle/_ref), compiled unmodified from its sources."""

    def __init__(self, threads: int | None = None):
        if not ref_available():
            raise FileNotFoundError("oracle/_ref not built (make -C oracle ref)")
        if threads is not None:
            os.environ["OMP_NUM_THREADS"] = str(threads)
        j = lambda n: os.path.join(REF_DIR, n)
        self.K = ct.CDLL(j("m5_kern_scalar.so"))
        self.E = ct.CDLL(j("m6_engine.so"))
        self.MT = ct.CDLL(j("m6_moe_tok.so"))
        self.G = ct.CDLL(j("m5_gemm.so"))
        self.FG = ct.CDLL(j("m5_gemm_fused.so"))
        self.B = ct.CDLL(j("m5_batch8_k.so"))
        self.K.m5_gemv.argtypes = [ct.c_int, _f, _u8, ct.c_int, ct.c_int, _f]
        self.K.m5_gemv.restype = ct.c_int
        self.E.m6_init_dl.argtypes = [ct.c_char_p] * 5
        self.E.m6_init_dl.restype = ct.c_int
        rc = self.E.m6_init_dl(*([j("m5_kern_scalar.so").encode()] * 5))
        assert rc == 0, rc
        self.E.m6_granite_moe.argtypes = [_f, _u64, _i, _f] + [ct.c_int] * 5 + [_f, _f]
        self.E.m6_granite_moe.restype = None
        self.E.m6_bailing_moe.argtypes = [_f, _u64, _i, _f, _f] + [ct.c_int] * 5 + [ct.c_float] + [ct.c_int] * 3 + [_f, _f]
        self.E.m6_bailing_moe.restype = None
        self.E.m6_granite_shexp.argtypes = [_f, _u64, _i, _f, _f, _f, _f, ct.c_int, ct.c_int]
        self.E.m6_granite_shexp.restype = None
        self.MT.m6_moe_tok.argtypes = [ct.c_void_p] * 8 + [ct.c_int] * 6 + [ct.c_void_p] * 3
        self.MT.m6_moe_tok.restype = None
        self.B.m5_gemvn_q4k.argtypes = [_f, ct.c_long, _u8, _i, ct.c_long, ct.c_int, ct.c_int, ct.c_int, _f]
        self.B.m5_gemvn_q4k.restype = ct.c_int
        self.B.m5_gemvn_q6k.argtypes = self.B.m5_gemvn_q4k.argtypes
        self.B.m5_gemvn_q6k.restype = ct.c_int
        self.dq_fp = ct.cast(self.G.m5_dequant_row, ct.c_void_p)
        self.ga_fp = ct.cast(self.FG.m5_gemm_auto, ct.c_void_p)
        self.nth = os.cpu_count() or 8

    def gemv(self, code, x, W, n_out, n_in):
        y = np.zeros(n_out, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        assert self.K.m5_gemv(code, pf(x), W.ctypes.data_as(_u8), n_out, n_in, pf(y)) == 0
        return y

    def decode(self, layer, x):
        ep, ec = layer.ptr_table()
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        out = np.zeros((x.shape[0], layer.hidden), np.float32)
        scratch = np.zeros(3 * layer.n_used * layer.inter + layer.n_used * layer.hidden, np.float32)
        gi = np.ascontiguousarray(layer.gate_inp, np.float32)
        for t in range(x.shape[0]):
            if layer.scoring == "softmax":
                self.E.m6_granite_moe(pf(x[t]), pu64(ep), pi(ec), pf(gi), layer.n_exp, layer.n_used,
                                      layer.inter, layer.hidden, layer.hidden, pf(scratch), pf(out[t]))
            else:
                pb = pf(layer.probs_b) if layer.probs_b is not None else None
                self.E.m6_bailing_moe(pf(x[t]), pu64(ep), pi(ec), pf(gi), pb, layer.n_exp,
                                      layer.n_used, layer.n_group, layer.n_group_used, layer.norm_w,
                                      ct.c_float(layer.w_scale), layer.inter, layer.hidden,
                                      layer.hidden, pf(scratch), pf(out[t]))
        return out

    def moe_tok(self, layer, X, order, wtop, fused=True):
        ep, ec = layer.ptr_table()
        X = np.ascontiguousarray(X, np.float32)
        T = X.shape[0]
        order = np.ascontiguousarray(order, np.int32)
        wtop = np.ascontiguousarray(wtop, np.float32)
        out = np.zeros((T, layer.hidden), np.float32)
        K, F, H = layer.n_used, layer.inter, layer.hidden
        work = np.empty(T * K * (H + 3 * F + H), np.float32)
        iwork = np.empty(T * K * 2 + layer.n_exp + 1, np.int32)
        wbuf = np.zeros(self.nth * 8208 * max(1, (max(H, F) + 8207) // 8208), np.float32)
        self.MT.m6_moe_tok(self.dq_fp, self.ga_fp if fused else None, wbuf.ctypes.data,
                           X.ctypes.data, order.ctypes.data, wtop.ctypes.data,
                           ep.ctypes.data, ec.ctypes.data, T, K, F, H, H, layer.n_exp,
                           out.ctypes.data, work.ctypes.data, iwork.ctypes.data)
        return out

    def shared_add(self, layer, X, out):
        """out[t] += the layer's ungated shared expert on X[t], computed by the reference's own
        m6_moe_tok with the shared expert as the only expert (order 0, weight 1: the combine's
        fused multiply-add then adds y exactly); the reference adds it in src/m6_engine.c:346."""
        X = np.ascontiguousarray(X, np.float32)
        T = X.shape[0]
        F, H = layer.shared_inter, layer.hidden
        ep = np.array([layer.sh_gate.ctypes.data, layer.sh_up.ctypes.data, layer.sh_down.ctypes.data], np.uint64)
        ec = np.array([layer.code_gu, layer.code_gu, layer.code_d], np.int32)
        order = np.zeros(T, np.int32)
        wtop = np.ones(T, np.float32)
        y = np.zeros((T, H), np.float32)
        work = np.empty(T * (H + 3 * F + H), np.float32)
        iwork = np.empty(T * 2 + 2, np.int32)
        wbuf = np.zeros(self.nth * 8208 * max(1, (max(H, F) + 8207) // 8208), np.float32)
        self.MT.m6_moe_tok(self.dq_fp, self.ga_fp, wbuf.ctypes.data, X.ctypes.data, order.ctypes.data,
                           wtop.ctypes.data, ep.ctypes.data, ec.ctypes.data, T, 1, F, H, H, 1,
                           y.ctypes.data, work.ctypes.data, iwork.ctypes.data)
        out += y
        return out

    def gemvn(self, code, x, x_stride, W, idx, per, n_out_e, n_in):
        idx = np.ascontiguousarray(idx, np.int32)
        y = np.zeros(len(idx) * n_out_e, np.float32)
        fn = self.B.m5_gemvn_q4k if code == 5 else self.B.m5_gemvn_q6k
        rc = fn(pf(np.ascontiguousarray(x, np.float32)), x_stride, W.ctypes.data_as(_u8), pi(idx),
                per, n_out_e, n_in, len(idx), pf(y))
        assert rc == 0, rc
        return y
