"""B200-native quantized MoE FFN layer (decode and chunked prefill) for Dracomancer's engine.

The product is the C-ABI library `libdraco_moe_b200.so` built from `csrc/` for sm_100a.  It
exports the reference engine's MoE entry points under their own names and signatures
(`m6_granite_moe`, `m6_bailing_moe`, `m6_moe_op`, `m6_granite_shexp`, `m6_moe_tok`,
`m5_gemvn_q4k/q6k`, `m5_gemv[_range]`, `m5_gemm*`, ...), so the reference's ctypes drivers
bind it in place of the CPU libraries, plus `draco_b200_*` extensions (whole-layer forward on
a token batch, routing only, activation mode, weight registry).

This module is the Python face of that library, mirroring how the reference's drivers call
it (`src/qwen35_engine.py:92-131`, `src/qwen35_prefill.py:65-83`, `src/k2_engine.py:97-106`):
`lib()` returns the ctypes handle with every signature declared, and a few helpers wrap the
common calls for numpy arrays and torch tensors.  There is no CPU fallback: when the library
is missing or no GPU is present the calls fail with an error.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

__all__ = ["lib", "LIB_PATH", "DracoMoeLayer", "M6MoeP", "layer_desc", "forward", "route", "granite_moe",
           "bailing_moe", "moe_tok", "last_error", "DracoError"]

PKG = os.path.dirname(os.path.abspath(__file__))
# DRACO_B200_LIB selects another build of the library (same ABI), e.g. one made with
# different compile-time tuning flags
LIB_PATH = os.environ.get("DRACO_B200_LIB") or os.path.join(PKG, "libdraco_moe_b200.so")

_f = ct.POINTER(ct.c_float)
_i = ct.POINTER(ct.c_int)
_u64 = ct.POINTER(ct.c_uint64)
_u8 = ct.POINTER(ct.c_uint8)
_i8 = ct.POINTER(ct.c_int8)
_i16 = ct.POINTER(ct.c_int16)
_i32 = ct.POINTER(ct.c_int32)
_vp = ct.c_void_p


class DracoError(RuntimeError):
    pass


class DracoMoeLayer(ct.Structure):
    """Layout of `DracoMoeLayer` in include/draco_moe_b200.h."""
    _fields_ = [("n_exp", ct.c_int), ("n_used", ct.c_int), ("inter", ct.c_int), ("n_in", ct.c_int),
                ("n_out", ct.c_int), ("exp_ptrs", _u64), ("exp_codes", _i), ("gate_inp", _vp),
                ("probs_b", _vp), ("scoring", ct.c_int), ("n_group", ct.c_int), ("n_group_used", ct.c_int),
                ("norm_w", ct.c_int), ("w_scale", ct.c_float), ("sh_gate", _vp), ("sh_up", _vp),
                ("sh_down", _vp), ("sh_code_g", ct.c_int), ("sh_code_u", ct.c_int), ("sh_code_d", ct.c_int),
                ("sh_ff", ct.c_int)]


class M6MoeP(ct.Structure):
    """Field order of the reference's M6MoeP (`src/m6_engine.c:306-316`)."""
    _fields_ = [("exp_ptrs", _u64), ("exp_codes", _i), ("gate_inp", _f), ("probs_b", _f),
                ("n_exp", ct.c_int), ("n_used", ct.c_int), ("n_group", ct.c_int), ("n_group_used", ct.c_int),
                ("norm_w", ct.c_int), ("w_scale", ct.c_float), ("inter", ct.c_int), ("n_in", ct.c_int),
                ("n_out", ct.c_int), ("sh_g", _vp), ("sh_u", _vp), ("sh_d", _vp), ("csg", ct.c_int),
                ("csu", ct.c_int), ("csd", ct.c_int), ("sh_ff", ct.c_int), ("scratch", _f)]


# name: (argtypes, restype) -- the reference drivers' own ctypes signatures where they exist
_SIGS = {
    "m6_granite_moe": ([_f, _u64, _i, _f] + [ct.c_int] * 5 + [_f, _f], None),
    "m6_bailing_moe": ([_f, _u64, _i, _f, _f] + [ct.c_int] * 5 + [ct.c_float] + [ct.c_int] * 3 + [_f, _f], None),
    "m6_moe_op": ([_f, _vp, _f], None),
    "m6_granite_shexp": ([_f, _u64, _i, _f, _f, _f, _f, ct.c_int, ct.c_int], None),
    "m6_moe_tok": ([_vp] * 8 + [ct.c_int] * 6 + [_vp] * 3, None),
    "m5_gemvn_q4k": ([_f, ct.c_long, _u8, _i, ct.c_long, ct.c_int, ct.c_int, ct.c_int, _f], ct.c_int),
    "m5_gemvn_q6k": ([_f, ct.c_long, _u8, _i, ct.c_long, ct.c_int, ct.c_int, ct.c_int, _f], ct.c_int),
    "m5_scalar_supported": ([ct.c_int], ct.c_int),
    "m5_gemv": ([ct.c_int, _f, _u8, ct.c_int, ct.c_int, _f], ct.c_int),
    "m5_gemv_range": ([ct.c_int, _f, _u8, ct.c_int, ct.c_int, _f, ct.c_int, ct.c_int], ct.c_int),
    "m5_dequant_row": ([ct.c_int, _u8, ct.c_int, _f], ct.c_int),
    "m5_gemm": ([ct.c_int, _vp, _vp, ct.c_int, ct.c_int, ct.c_int, _vp, _vp], ct.c_int),
    "m5_gemm_auto": ([ct.c_int, _vp, _vp, ct.c_int, ct.c_int, ct.c_int, _vp], ct.c_int),
    "m5_gemm_q80": ([_f, _u8, ct.c_int, ct.c_int, ct.c_int, _f], None),
    "m5_gemm_q6k": ([_f, _u8, ct.c_int, ct.c_int, ct.c_int, _f], None),
    "m5_gemm_q4k": ([_f, _u8, ct.c_int, ct.c_int, ct.c_int, _f], None),
    "m6_init_dl": ([ct.c_char_p] * 5, ct.c_int),
    "m6_set_moe_chunk": ([ct.c_int], ct.c_int),
    "m6_prof_reset": ([], None),
    "m6_prof_get": ([ct.c_int], ct.c_double),
    "m6_prof_cnt": ([ct.c_int], ct.c_long),
    "m6_rowbytes": ([ct.c_int, ct.c_int], ct.c_size_t),
    "draco_b200_last_error": ([], ct.c_char_p),
    "draco_b200_version": ([], ct.c_char_p),
    "draco_b200_device_count": ([], ct.c_int),
    "draco_b200_moe_forward": ([ct.POINTER(DracoMoeLayer), _vp, ct.c_int, _vp, _vp, _vp, _vp], ct.c_int),
    "draco_b200_route": ([ct.POINTER(DracoMoeLayer), _vp, ct.c_int, _vp, _vp, _vp], ct.c_int),
    "draco_b200_experts_forward": ([ct.POINTER(DracoMoeLayer), _vp, ct.c_int, _vp, _vp, ct.c_int, ct.c_int, _vp,
                                    ct.c_int, ct.c_int, _vp], ct.c_int),
    "draco_b200_experts_forward_to_ranks": ([ct.POINTER(DracoMoeLayer), _vp, ct.c_int, _vp, _vp, ct.c_int, ct.c_int,
                                             _vp, ct.c_int, ct.c_int, _vp], ct.c_int),
    "draco_b200_ep_plan": ([_vp, ct.c_int, ct.c_int, ct.c_int, ct.c_int, ct.c_int, _vp, _vp, _vp, _vp], ct.c_int),
    "draco_b200_ep_pack": ([_vp, _vp, _vp, _vp, ct.c_int, _vp, ct.c_int, ct.c_int, ct.c_int, ct.c_int, _vp, _vp,
                            _vp], ct.c_int),
    "draco_b200_ep_combine": ([_vp, _vp, ct.c_int, ct.c_int, ct.c_int, _vp, _vp, _vp], ct.c_int),
    "draco_b200_ep_mem_alloc": ([ct.c_size_t, ct.POINTER(ct.c_void_p), _vp], ct.c_int),
    "draco_b200_ep_mem_open": ([_vp, ct.POINTER(ct.c_void_p)], ct.c_int),
    "draco_b200_ep_mem_close": ([_vp], ct.c_int),
    "draco_b200_ep_mem_free": ([_vp], ct.c_int),
    "draco_b200_ep_push": ([_vp, _vp, _vp, _vp, ct.c_int, ct.c_int, _vp, ct.c_int, ct.c_int, ct.c_int, _vp, ct.c_int,
                            _vp, _vp], ct.c_int),
    "draco_b200_ep_barrier": ([_vp, _vp, _vp, ct.c_int, ct.c_int, _vp, _vp], ct.c_int),
    "draco_b200_ep_pull_combine": ([_vp, _vp, ct.c_int, ct.c_int, ct.c_int, ct.c_int, ct.c_int, _vp, _vp, _vp],
                                   ct.c_int),
    "draco_b200_set_act_mode": ([ct.c_int], ct.c_int),
    "draco_b200_set_gemm_path": ([ct.c_int], ct.c_int),
    "draco_b200_set_fused_decode": ([ct.c_int], ct.c_int),
    "draco_b200_test_fused_barrier_extra": ([ct.c_int], ct.c_int),
    "draco_b200_profile": ([ct.c_int], ct.c_int),
    "draco_b200_profile_read": ([ct.POINTER(ct.c_double), ct.POINTER(ct.c_long), ct.c_int], ct.c_int),
    "draco_b200_launch_count": ([], ct.c_long),
    "draco_b200_register": ([_vp, ct.c_size_t], ct.c_int),
    "draco_b200_forget": ([_vp], ct.c_int),
    "draco_b200_reset": ([], None),
    "draco_b200_registered_bytes": ([], ct.c_size_t),
    "draco_b200_expf": ([_f, _f, ct.c_long], ct.c_int),
    "draco_b200_router_logits": ([_f, _f, ct.c_int, ct.c_int, ct.c_int, _f], ct.c_int),
    "draco_b200_q8k_quantize": ([_f, ct.c_int, _f, _i8, _i16], ct.c_int),
    "draco_b200_q8k_block_dots": ([ct.c_int, _u8, ct.c_int, ct.c_int, _i8, _i16, _i32], ct.c_int),
    "draco_b200_gemv_q8k": ([ct.c_int, _u8, ct.c_int, ct.c_int, _i8, _f, _i16, _f], ct.c_int),
}

_LIB = None


def lib() -> ct.CDLL:
    """The loaded library with every signature declared.  Raises if it was never built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise DracoError(f"{LIB_PATH} is missing: build it with `python -m dracomancer_llmengine_b200.build`")
        L = ct.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


PHASES = ("route", "dispatch", "gateup", "down", "shared", "combine", "gather", "fused")


def profile(enable: bool) -> None:
    lib().draco_b200_profile(1 if enable else 0)


def profile_read() -> dict:
    """{phase: (total_ms, launches)} of the per-phase CUDA-event timing."""
    ms = (ct.c_double * len(PHASES))()
    n = (ct.c_long * len(PHASES))()
    lib().draco_b200_profile_read(ms, n, len(PHASES))
    return {p: (ms[i], n[i]) for i, p in enumerate(PHASES)}


def last_error() -> str:
    return (lib().draco_b200_last_error() or b"").decode()


def _check(rc: int, what: str):
    if rc != 0:
        raise DracoError(f"{what} failed ({rc}): {last_error()}")


def _ptr(a) -> int:
    """Address of a numpy array or torch tensor (host or device)."""
    if a is None:
        return 0
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def layer_desc(layer, keep: list) -> DracoMoeLayer:
    """DracoMoeLayer for a synth.MoELayer-like object (numpy weight buffers); arrays that must
    outlive the call are appended to `keep`."""
    ep, ec = layer.ptr_table()
    gi = np.ascontiguousarray(layer.gate_inp, np.float32)
    keep += [ep, ec, gi]
    d = DracoMoeLayer()
    d.n_exp, d.n_used, d.inter = layer.n_exp, layer.n_used, layer.inter
    d.n_in = d.n_out = layer.hidden
    d.exp_ptrs = ep.ctypes.data_as(_u64)
    d.exp_codes = ec.ctypes.data_as(_i)
    d.gate_inp = gi.ctypes.data
    if layer.probs_b is not None:
        pb = np.ascontiguousarray(layer.probs_b, np.float32)
        keep.append(pb)
        d.probs_b = pb.ctypes.data
    d.scoring = 0 if layer.scoring == "softmax" else 1
    d.n_group, d.n_group_used, d.norm_w = layer.n_group, layer.n_group_used, layer.norm_w
    d.w_scale = layer.w_scale
    if layer.shared_inter:
        d.sh_gate, d.sh_up, d.sh_down = layer.sh_gate.ctypes.data, layer.sh_up.ctypes.data, layer.sh_down.ctypes.data
        d.sh_code_g = d.sh_code_u = layer.code_gu
        d.sh_code_d = layer.code_d
        d.sh_ff = layer.shared_inter
    keep.append(d)
    return d


def forward(layer, X, out=None, order_out=None, wtop_out=None, stream=None):
    """Whole layer (routing, experts, combine, shared expert) on a token batch X [T, hidden].
    numpy in -> numpy out (synchronous); torch CUDA tensors in -> written in place."""
    keep: list = []
    d = layer_desc(layer, keep)
    is_np = isinstance(X, np.ndarray)
    if is_np:
        X = np.ascontiguousarray(X, np.float32)
        T = X.shape[0]
        if out is None:
            out = np.empty((T, layer.hidden), np.float32)
    else:
        T = X.shape[0]
        assert out is not None
    st = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
    rc = lib().draco_b200_moe_forward(ct.byref(d), _ptr(X), T, _ptr(out), _ptr(order_out), _ptr(wtop_out), st)
    _check(rc, "draco_b200_moe_forward")
    return out


def route(layer, X):
    """(order int32[T, K], wtop fp32[T, K]) from the device router."""
    keep: list = []
    d = layer_desc(layer, keep)
    X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
    T = X.shape[0]
    order = np.empty((T, layer.n_used), np.int32)
    wtop = np.empty((T, layer.n_used), np.float32)
    _check(lib().draco_b200_route(ct.byref(d), X.ctypes.data, T, order.ctypes.data, wtop.ctypes.data, None),
           "draco_b200_route")
    return order, wtop


def granite_moe(layer, x):
    """m6_granite_moe on one token (reference call shape of src/qwen35_engine.py:300)."""
    ep, ec = layer.ptr_table()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(layer.hidden, np.float32)
    gi = np.ascontiguousarray(layer.gate_inp, np.float32)
    lib().m6_granite_moe(x.ctypes.data_as(_f), ep.ctypes.data_as(_u64), ec.ctypes.data_as(_i),
                         gi.ctypes.data_as(_f), layer.n_exp, layer.n_used, layer.inter, layer.hidden,
                         layer.hidden, None, out.ctypes.data_as(_f))
    return out


def bailing_moe(layer, x):
    """m6_bailing_moe on one token."""
    ep, ec = layer.ptr_table()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(layer.hidden, np.float32)
    gi = np.ascontiguousarray(layer.gate_inp, np.float32)
    pb = None if layer.probs_b is None else np.ascontiguousarray(layer.probs_b, np.float32)
    lib().m6_bailing_moe(x.ctypes.data_as(_f), ep.ctypes.data_as(_u64), ec.ctypes.data_as(_i),
                         gi.ctypes.data_as(_f), None if pb is None else pb.ctypes.data_as(_f), layer.n_exp,
                         layer.n_used, layer.n_group, layer.n_group_used, layer.norm_w,
                         ct.c_float(layer.w_scale), layer.inter, layer.hidden, layer.hidden, None,
                         out.ctypes.data_as(_f))
    return out


def moe_tok(layer, X, order, wtop):
    """m6_moe_tok with caller routing (reference call shape of src/qwen35_prefill.py:195-197)."""
    ep, ec = layer.ptr_table()
    X = np.ascontiguousarray(X, np.float32)
    order = np.ascontiguousarray(order, np.int32)
    wtop = np.ascontiguousarray(wtop, np.float32)
    T = X.shape[0]
    out = np.empty((T, layer.hidden), np.float32)
    lib().m6_moe_tok(None, None, None, X.ctypes.data, order.ctypes.data, wtop.ctypes.data, ep.ctypes.data,
                     ec.ctypes.data, T, layer.n_used, layer.inter, layer.hidden, layer.hidden, layer.n_exp,
                     out.ctypes.data, None, None)
    return out
