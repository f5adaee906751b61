"""The allocation-free entry point draco_b200_moe_tok_noalloc, for callers that cannot let a
library allocate device memory (an engine that reserves HBM for weights and KV cache up front
and forbids allocations outside its pool, or a decode loop that cannot afford cudaMalloc's
implicit synchronisation).  It keeps its scratch in a fixed-size device array inside the
library, so the caller passes only inputs and outputs (all device memory).

Checked through the C ABI against the CPU oracle (the C restatement of src/m6_moe_tok.c, pinned
to the reference) and against the existing entry point m6_moe_tok, with the tolerance the other
parity tests use, on two calls in a row (the shared scratch keeps the first call's contents; the
second call must not depend on them).  The calls cover the single-block dispatch (few
assignments) and the multi-chunk dispatch (more than 1024 assignments, whose per-chunk counts
live in the shared scratch), Q4_K/Q6_K and Q8_0 layers, and the device's free memory across a
call.  This file sorts last so that a run stopping at the first failure has already run every
other test.
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


def _device_table(torch, layer, dev):
    """Expert weights copied to device memory owned by the caller; the table of their device
    addresses (gate, up, down per expert) and the format codes."""
    g = torch.from_numpy(layer.gate).to(dev)
    u = torch.from_numpy(layer.up).to(dev)
    d = torch.from_numpy(layer.down).to(dev)
    E = layer.n_exp
    ep_dev = np.zeros(3 * E, np.uint64)
    ep_dev[0::3] = g.data_ptr() + layer.gate.shape[1] * np.arange(E, dtype=np.uint64)
    ep_dev[1::3] = u.data_ptr() + layer.up.shape[1] * np.arange(E, dtype=np.uint64)
    ep_dev[2::3] = d.data_ptr() + layer.down.shape[1] * np.arange(E, dtype=np.uint64)
    _, ec = layer.ptr_table()
    return (g, u, d), ep_dev, ec


@pytest.mark.parametrize("codes", [(synth.CODE_Q4_K, synth.CODE_Q6_K), (synth.CODE_Q8_0, synth.CODE_Q8_0)],
                         ids=["q4k_q6k", "q8_0"])
def test_noalloc_matches_oracle_two_calls(port, codes):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU test without a CUDA device")
    fn = _bind()
    dev = torch.device("cuda", 0)
    layer = synth.make_layer(hidden=2048, n_exp=32, n_used=8, inter=768, seed=77, code_gu=codes[0], code_d=codes[1])
    keep, ep_dev, ec = _device_table(torch, layer, dev)
    E = layer.n_exp
    stream = torch.cuda.current_stream(dev)
    # 24 tokens: 192 assignments (one-block dispatch); 200 tokens: 1600 (multi-chunk dispatch)
    for call, T in enumerate((24, 200)):
        X = synth.make_tokens(layer, T, 77 + call)
        order, wtop = port.route(layer, X)
        want = port.moe_tok(layer, X, order, wtop)          # the oracle
        ref = dm.moe_tok(layer, X, order, wtop)             # the existing entry point
        assert T * layer.n_used * (layer.inter + layer.hidden) * 4 < SCRATCH_MAX
        Xd = torch.from_numpy(X).to(dev)
        od = torch.from_numpy(order).to(dev)
        wd = torch.from_numpy(wtop).to(dev)
        out = torch.full((T, layer.hidden), float("nan"), device=dev)
        args = (Xd.data_ptr(), od.data_ptr(), wd.data_ptr(), ep_dev.ctypes.data, ec.ctypes.data, T, layer.n_used,
                layer.inter, layer.hidden, layer.hidden, E, out.data_ptr(), stream.cuda_stream)
        assert fn(*args) == 0
        torch.cuda.synchronize()
        if call == 1:
            # a repeated call allocates nothing: the device's free memory is unchanged across it
            free0 = torch.cuda.mem_get_info(dev)[0]
            assert fn(*args) == 0
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info(dev)[0] == free0
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        err = _rel(got, want)
        assert err <= REL_L2_TOL, ("oracle", call, err)
        assert _rel(got, ref) <= REL_L2_TOL, ("m6_moe_tok", call)
    del keep


def test_noalloc_rejects_sizes_beyond_its_maximum():
    torch = pytest.importorskip("torch")
    fn = _bind()
    layer = synth.make_layer(hidden=2048, n_exp=32, n_used=8, inter=768, seed=78, weights=False)
    _, ec = layer.ptr_table()
    ec[:] = np.tile(np.array([5, 5, 4], np.int32), layer.n_exp)
    ep_dev = np.full(3 * layer.n_exp, 1 << 20, np.uint64)   # aligned, never read
    # act + y per assignment = (768 + 2048) * 4 bytes: 4096 tokens x 8 is ~369 MB > 32 MiB
    T = 4096
    assert T * 8 * (768 + 2048) * 4 > SCRATCH_MAX
    dummy = torch.zeros(16, device="cuda")
    rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), ep_dev.ctypes.data, ec.ctypes.data, T, 8, 768,
            2048, 2048, layer.n_exp, dummy.data_ptr(), None)
    assert rc == -4


def test_noalloc_rejects_misaligned_weight_addresses():
    """A table entry the row decoders cannot read (odd address, Q4_K off 16 bytes, null) is
    refused with -1 before anything is launched."""
    torch = pytest.importorskip("torch")
    fn = _bind()
    E = 16
    ec = np.tile(np.array([5, 5, 4], np.int32), E)
    dummy = torch.zeros(16, device="cuda")
    for bad_index, bad_value in ((0, (1 << 20) + 8), (2, (1 << 20) + 1), (4, 0)):
        ep_dev = np.full(3 * E, 1 << 20, np.uint64)
        ep_dev[bad_index] = bad_value
        rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), ep_dev.ctypes.data, ec.ctypes.data, 4, 8, 768,
                2048, 2048, E, dummy.data_ptr(), None)
        assert rc == -1, (bad_index, bad_value)
