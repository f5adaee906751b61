"""The fused single-launch decode layer (decode.cu fused_decode_kernel): batches of at most 8
tokens and 64 token-expert assignments run router logits, selection, gate/up + SwiGLU, down,
the k-ordered combine and the shared expert as one cooperative kernel.

Checked against the CPU oracle (routing bit-exact, output rel-L2 <= 1e-3, the bars of the other
parity tests), against the separate-kernel path it replaces, with caller-given routing
(m6_moe_tok), with a shared expert, and for its bounded grid-barrier wait: a barrier that waits
for one block more than the grid gives up after about a second, the call reports -5, and the
next call on the same device is correct again.
"""
import ctypes as ct

import numpy as np
import pytest

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def forward_with_routing(layer, X):
    T = X.shape[0]
    order = np.empty((T, layer.n_used), np.int32)
    wtop = np.empty((T, layer.n_used), np.float32)
    out = dm.forward(layer, X, order_out=order, wtop_out=wtop)
    return out, order, wtop


LAYERS = {
    "cfg1_shape_softmax": dict(hidden=2048, n_exp=128, n_used=8, inter=768, seed=41),
    "groups_bias_shared": dict(hidden=2048, n_exp=64, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                               n_group_used=4, w_scale=2.5, bias=True, shared_inter=512, seed=42),
    "k2_rows_shared": dict(hidden=7168, n_exp=32, n_used=8, inter=2048, scoring="sigmoid", w_scale=2.827,
                           bias=True, shared_inter=2048, seed=43),
    "e384_sigmoid": dict(hidden=512, n_exp=384, n_used=8, inter=256, scoring="sigmoid", w_scale=2.827,
                         bias=True, seed=45),
}


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("T", [1, 3, 8])
def test_fused_decode_matches_oracle(dlib, port, name, T):
    layer = synth.make_layer(**LAYERS[name])
    X = synth.make_tokens(layer, T, 100 + T)
    dm.profile(True)
    out, order, wtop = forward_with_routing(layer, X)
    prof = dm.profile_read()
    dm.profile(False)
    assert prof["fused"][1] >= 1, "the fused kernel did not run"
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(order, o_ref), "routing indices differ"
    assert np.array_equal(bits(wtop), bits(w_ref)), "gate weights differ in bits"
    ref = port.layer_forward(layer, X, o_ref, w_ref)
    err = rel_l2(out, ref)
    assert err <= REL_L2_TOL, err


def test_fused_equals_separate_kernels(dlib):
    """The fused kernel and the separate kernels it replaces compute the same sums in the same
    order: identical outputs."""
    layer = synth.make_layer(**LAYERS["groups_bias_shared"])
    X = synth.make_tokens(layer, 5, 7)
    a = dm.forward(layer, X)
    prev = dlib.draco_b200_set_fused_decode(0)
    try:
        b = dm.forward(layer, X)
    finally:
        dlib.draco_b200_set_fused_decode(prev)
    assert np.array_equal(bits(a), bits(b))


def test_fused_given_routing(dlib, port):
    """m6_moe_tok with caller routing (ids outside the table are skipped) on a decode batch."""
    layer = synth.make_layer(**LAYERS["cfg1_shape_softmax"])
    X = synth.make_tokens(layer, 4, 9)
    order, wtop = port.route(layer, X)
    order = order.copy()
    order[1, 3] = -1          # no expert: skipped by both
    got = dm.moe_tok(layer, X, order, wtop)
    want = port.moe_tok(layer, X, order, wtop)
    assert rel_l2(got, want) <= REL_L2_TOL


@pytest.mark.parametrize("shared", [False, True])
def test_fused_no_routed_expert(dlib, port, shared):
    """Every routing entry names no expert (ids -1): no routed expert runs; the output is zero,
    or the shared expert alone."""
    kw = dict(LAYERS["cfg1_shape_softmax"])
    if shared:
        kw["shared_inter"] = 512
    layer = synth.make_layer(**kw)
    X = synth.make_tokens(layer, 3, 12)
    order = np.full((3, layer.n_used), -1, np.int32)
    wtop = np.ones((3, layer.n_used), np.float32)
    keep: list = []
    d = dm.layer_desc(layer, keep)
    got = np.full((3, layer.hidden), np.nan, np.float32)
    dm.profile(True)
    rc = dlib.draco_b200_experts_forward(ct.byref(d), X.ctypes.data, 3, order.ctypes.data, wtop.ctypes.data, 0, 0,
                                         got.ctypes.data, 1 if shared else 0, 0, None)
    prof = dm.profile_read()
    dm.profile(False)
    assert rc == 0, dm.last_error()
    assert prof["fused"][1] >= 1, "the fused kernel did not run"
    if shared:
        want = port.layer_forward(layer, X, order, wtop)
        assert rel_l2(got, want) <= REL_L2_TOL
    else:
        assert not np.any(got)


def test_fused_ties_lower_index(dlib, port):
    layer = synth.make_layer(hidden=2048, n_exp=64, n_used=8, inter=512, seed=44)
    layer.gate_inp[1::2] = layer.gate_inp[0::2]     # experts 2k and 2k+1 tie everywhere
    X = synth.make_tokens(layer, 6, 44)
    out, order, wtop = forward_with_routing(layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(order, o_ref)
    assert np.array_equal(bits(wtop), bits(w_ref))
    assert rel_l2(out, port.layer_forward(layer, X, o_ref, w_ref)) <= REL_L2_TOL


def test_fused_barrier_wait_runs_out_and_reports(dlib, port):
    """A grid barrier that waits for one arrival more than the grid has blocks gives up after its
    limit (about a second): the call returns -5 and the device stays usable."""
    layer = synth.make_layer(**LAYERS["cfg1_shape_softmax"])
    X = synth.make_tokens(layer, 2, 11)
    keep: list = []
    d = dm.layer_desc(layer, keep)
    out = np.empty((2, layer.hidden), np.float32)
    dlib.draco_b200_test_fused_barrier_extra(1)
    dm.profile(True)
    try:
        rc = dlib.draco_b200_moe_forward(ct.byref(d), X.ctypes.data, 2, out.ctypes.data, None, None, None)
    finally:
        dlib.draco_b200_test_fused_barrier_extra(0)
        prof = dm.profile_read()
        dm.profile(False)
    assert prof["fused"][1] >= 1, "the fused kernel did not run"
    assert rc == -5, (rc, dm.last_error(), prof["fused"])
    assert "0x1000" in dm.last_error()
    good = dm.forward(layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert rel_l2(good, port.layer_forward(layer, X, o_ref, w_ref)) <= REL_L2_TOL
