"""Routing with the numpy K2 drivers' renormalisation (norm_w = 2), checked on the CPU.

src/k2_engine.py:500-508 (decode) and src/k2_prefill.py:122-127 (prefill) select with the
sigmoid scores plus bias and weight with the plain scores, then renormalise with numpy:
`rw = rw / rw.sum() * R_SCALING` -- no 6.1e-5 clamp, and numpy's float32 sum, which adds 8
running partial sums for 8 or more values.  The restatement (oracle/moe_oracle.c, norm_w = 2) is
checked here bit-for-bit against numpy itself applied to the same scores; the GPU router is
checked bit-for-bit against the restatement in tests/test_gpu_parity.py.  (The drivers' logits
come from BLAS and their exp from numpy; both are outside what the C path reproduces, so the
scores here are the C path's.)
"""
import numpy as np
import pytest

from dracomancer_llmengine_b200 import synth


def numpy_weights(P, idx, scale):
    rw = np.take_along_axis(P, idx, 1)
    return (rw / rw.sum(1, keepdims=True) * scale).astype(np.float32)


@pytest.mark.parametrize("n_used,n_exp,scale", [(8, 384, 2.827), (12, 96, 2.5), (6, 64, 1.0), (20, 128, 2.5)])
def test_k2_driver_renorm_matches_numpy(port, n_used, n_exp, scale):
    layer = synth.make_layer(hidden=512, n_exp=n_exp, n_used=n_used, inter=256, scoring="sigmoid", w_scale=scale,
                             bias=True, seed=n_used + n_exp, weights=False)
    X = synth.make_tokens(layer, 64, 5)
    layer.norm_w = 1
    i1, w1, P = port.route_probs(layer, X)
    layer.norm_w = 2
    i2, w2, _ = port.route_probs(layer, X)
    assert np.array_equal(i1, i2), "the renormalisation must not change the selection"
    want = numpy_weights(P, i2, scale if scale not in (0.0, 1.0) else 1.0)
    assert np.array_equal(w2.view(np.uint32), want.view(np.uint32))
    # the batched router gives the same bits
    ib, wb = port.route(layer, X)
    assert np.array_equal(ib, i2) and np.array_equal(wb.view(np.uint32), w2.view(np.uint32))


def test_pairwise_sum_is_numpys(port):
    import ctypes as ct
    L = port.L
    L.orc_pairwise_sum.argtypes = [ct.POINTER(ct.c_float), ct.c_int]
    L.orc_pairwise_sum.restype = ct.c_float
    rng = np.random.default_rng(3)
    for n in range(1, 65):
        for _ in range(50):
            a = (rng.random(n) * rng.choice([1e-4, 1.0, 1e4], n)).astype(np.float32)
            got = L.orc_pairwise_sum(a.ctypes.data_as(ct.POINTER(ct.c_float)), n)
            assert np.float32(got) == a.sum(), n
