"""Regenerate the golden fixtures from the reference's own C (oracle/_ref, compiled from the
reference sources by `make -C oracle ref`).  Run in a container that has the reference:

    python tests/golden/make_golden.py

For each case of gen.CASES it stores the reference outputs of
  * the decode layer entry point (m6_granite_moe / m6_bailing_moe, src/m6_layer.c:771-873),
  * the scalar row kernel m5_gemv on expert 0's gate and down matrices (src/m5_kern_scalar.c),
  * the chunked-prefill m6_moe_tok (src/m6_moe_tok.c) with its fused GEMM, on routing made by
    the reference's numpy router (src/qwen35_prefill.py:180-188, softmax) or the K2 numpy
    router (src/k2_engine.py:500-508, sigmoid), stored with the fixture.
Inputs are rebuilt from the seed by gen.py, so only outputs (and the routing) are stored.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import gen  # noqa: E402
from oracle.oracle import Ref  # noqa: E402


def numpy_router(layer, X):
    lg = X @ layer.gate_inp.T
    K = layer.n_used
    if layer.scoring == "softmax":
        lg = lg - lg.max(1, keepdims=True)
        P = np.exp(lg)
        P /= P.sum(1, keepdims=True)
        order = np.argsort(-P, axis=1, kind="stable")[:, :K]
        w = np.take_along_axis(P, order, 1)
        w /= np.maximum(w.sum(1, keepdims=True), 6.103515625e-5)
    else:
        P = 1.0 / (1.0 + np.exp(-lg))
        sel = P + (layer.probs_b if layer.probs_b is not None else 0.0)
        order = np.argsort(-sel, axis=1, kind="stable")[:, :K]
        w = np.take_along_axis(P, order, 1)
        w = w / w.sum(1, keepdims=True) * (layer.w_scale if layer.w_scale not in (0.0, 1.0) else 1.0)
    return np.ascontiguousarray(order, np.int32), np.ascontiguousarray(w, np.float32)


def main():
    R = Ref(threads=1)
    for name, (kw, T) in gen.CASES.items():
        layer = gen.Layer(**kw)
        X = gen.tokens(kw["seed"], T, layer.hidden)
        dec = R.decode(layer, X)
        gv_gate = R.gemv(layer.code_gu, X[0], layer.gate[0], layer.inter, layer.hidden)
        gv_down = R.gemv(layer.code_d, X[0][:layer.inter].copy(), layer.down[0], layer.hidden, layer.inter)
        order, wtop = numpy_router(layer, X)
        tok = R.moe_tok(layer, X, order, wtop)
        np.savez(os.path.join(HERE, f"{name}.npz"), decode=dec, gemv_gate=gv_gate, gemv_down=gv_down,
                 order=order, wtop=wtop, moe_tok=tok)
        print(name, dec.shape, tok.shape)


if __name__ == "__main__":
    main()
