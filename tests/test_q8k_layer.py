"""The whole layer in Q8_K activation mode (draco_b200_set_act_mode(1)).

In this mode the gate/up products take each token row quantised to Q8_K (per 256 values: an fp32
scale d and int8 codes q) and run as integer superblock dots; routing and the down products stay
fp32.  The reference has no Q8_K path, so the check feeds the reference's own C (oracle/_ref
m6_moe_tok) the dequantised rows x_hat = d * q for its gate/up input, with the routing computed
from the unquantised rows (as the device does):

  * routing: bit-exact against the CPU restatement of the C router on x;
  * layer output: the integer dots equal the fp32 dots of w and x_hat up to float rounding, so the
    outputs agree to rel-L2 <= 1e-5 (measured ~1e-7);
  * against the fp32 layer on x the difference is the activation quantisation (reported, bounded
    loosely by 2e-2).
"""
import numpy as np
import pytest

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu

Q8K_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dequant_rows(port, X):
    """x_hat = d * q per 256-value block, row by row (the Q8_K restatement of the oracle)."""
    out = np.empty_like(X)
    for t in range(X.shape[0]):
        d, q, _ = port.q8k_quantize(X[t])
        out[t] = (np.repeat(d, 256) * q.astype(np.float32)).astype(np.float32)
    return out


def forward_q8k(dlib, layer, X):
    prev = dlib.draco_b200_set_act_mode(1)
    try:
        order = np.empty((X.shape[0], layer.n_used), np.int32)
        wtop = np.empty((X.shape[0], layer.n_used), np.float32)
        out = dm.forward(layer, X, order_out=order, wtop_out=wtop)
    finally:
        dlib.draco_b200_set_act_mode(prev)
    return out, order, wtop


LAYERS = {
    "softmax_q4k_q6k": dict(hidden=2048, n_exp=64, n_used=8, inter=512, seed=81),
    "sigmoid_groups": dict(hidden=1024, n_exp=64, n_used=8, inter=512, scoring="sigmoid", n_group=8,
                           n_group_used=4, w_scale=2.5, bias=True, seed=82),
    "q6k_gate_up": dict(hidden=1024, n_exp=32, n_used=4, inter=256, code_gu=synth.CODE_Q6_K, seed=83),
}


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("T", [1, 7, 96])
def test_q8k_layer_matches_reference_on_dequantised_rows(dlib, port, ref, name, T):
    layer = synth.make_layer(**LAYERS[name])
    X = synth.make_tokens(layer, T, 200 + T)
    out, order, wtop = forward_q8k(dlib, layer, X)
    o_ref, w_ref = port.route(layer, X)
    assert np.array_equal(order, o_ref), "routing indices differ"
    assert np.array_equal(wtop.view(np.uint32), w_ref.view(np.uint32)), "gate weights differ in bits"
    want = ref.moe_tok(layer, dequant_rows(port, X), o_ref, w_ref)
    err = rel_l2(out, want)
    assert err <= Q8K_TOL, err
    # the quantisation itself, against the fp32 layer (informative bound)
    assert rel_l2(out, ref.moe_tok(layer, X, o_ref, w_ref)) <= 2e-2
