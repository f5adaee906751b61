"""The allocation-free entry point draco_b200_moe_tok_noalloc, for callers that cannot let a
library allocate device memory (an engine that reserves HBM for weights and KV cache up front
and forbids allocations outside its pool, or a decode loop that cannot afford cudaMalloc's
implicit synchronisation).  It keeps its scratch in a fixed-size device array inside the
library, so the caller passes only inputs and outputs (all device memory).

Checked through the C ABI against the existing entry point m6_moe_tok on the same inputs,
with the tolerance the other parity tests use, on two calls in a row (the shared scratch keeps
the first call's contents; the second call must not depend on them).  This file sorts last so
that a run stopping at the first failure has already run every other test.
"""
import ctypes as ct

import numpy as np
import pytest

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3
SCRATCH_MAX = 32 << 20     # the entry point's fixed scratch size


def _bind():
    L = dm.lib()
    fn = L.draco_b200_moe_tok_noalloc
    fn.argtypes = [ct.c_void_p] * 5 + [ct.c_int] * 6 + [ct.c_void_p, ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def test_noalloc_matches_moe_tok_two_calls():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU test without a CUDA device")
    fn = _bind()
    dev = torch.device("cuda", 0)
    layer = synth.make_layer(hidden=2048, n_exp=32, n_used=8, inter=768, seed=77)
    # expert weights in device memory owned by the caller; the table holds device addresses
    g = torch.from_numpy(layer.gate).to(dev)
    u = torch.from_numpy(layer.up).to(dev)
    d = torch.from_numpy(layer.down).to(dev)
    E = layer.n_exp
    ep_dev = np.zeros(3 * E, np.uint64)
    ep_dev[0::3] = g.data_ptr() + layer.gate.shape[1] * np.arange(E, dtype=np.uint64)
    ep_dev[1::3] = u.data_ptr() + layer.up.shape[1] * np.arange(E, dtype=np.uint64)
    ep_dev[2::3] = d.data_ptr() + layer.down.shape[1] * np.arange(E, dtype=np.uint64)
    _, ec = layer.ptr_table()
    stream = torch.cuda.current_stream(dev)
    for call, T in enumerate((24, 9)):
        X = synth.make_tokens(layer, T, 77 + call)
        order, wtop = dm.route(layer, X)
        ref = dm.moe_tok(layer, X, order, wtop)            # the existing entry point
        Xd = torch.from_numpy(X).to(dev)
        od = torch.from_numpy(order).to(dev)
        wd = torch.from_numpy(wtop).to(dev)
        out = torch.full((T, layer.hidden), float("nan"), device=dev)
        rc = fn(Xd.data_ptr(), od.data_ptr(), wd.data_ptr(), ep_dev.ctypes.data, ec.ctypes.data, T, layer.n_used,
                layer.inter, layer.hidden, layer.hidden, E, out.data_ptr(), stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        err = _rel(got, ref)
        assert err <= REL_L2_TOL, (call, err)


def test_noalloc_rejects_sizes_beyond_its_maximum():
    torch = pytest.importorskip("torch")
    fn = _bind()
    layer = synth.make_layer(hidden=2048, n_exp=32, n_used=8, inter=768, seed=78, weights=False)
    _, ec = layer.ptr_table()
    ec[:] = np.tile(np.array([5, 5, 4], np.int32), layer.n_exp)
    ep_dev = np.zeros(3 * layer.n_exp, np.uint64)
    # act + y per assignment = (768 + 2048) * 4 bytes: 4096 tokens x 8 is ~369 MB > 32 MiB
    T = 4096
    assert T * 8 * (768 + 2048) * 4 > SCRATCH_MAX
    dummy = torch.zeros(16, device="cuda")
    rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), ep_dev.ctypes.data, ec.ctypes.data, T, 8, 768,
            2048, 2048, layer.n_exp, dummy.data_ptr(), None)
    assert rc == -4
