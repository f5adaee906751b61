"""The layer called on host buffers, page-locked (the copies and launches captured once and
replayed as a graph) and pageable, and on device buffers:

  * all three give bit-identical outputs, expert indices and gate weights, also on the graph's
    replay;
  * the routing is bit-exact against the C restatement of the reference routers and the output
    within rel-L2 1e-3 of the oracle layer.
Token counts 100, 301 and 1030 (ragged against every tile size).
"""
import ctypes as ct

import numpy as np
import pytest
import torch

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu

LAYERS = {
    "softmax": dict(hidden=1024, n_exp=64, n_used=8, inter=256, seed=71),
    "sigmoid_groups_shared": dict(hidden=1024, n_exp=64, n_used=6, inter=256, scoring="sigmoid", n_group=8,
                                  n_group_used=4, w_scale=2.5, bias=True, shared_inter=256, seed=72),
}


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def call(L, desc, X, T, out, order, wtop, stream=None):
    rc = L.draco_b200_moe_forward(ct.byref(desc), X.data_ptr(), T, out.data_ptr(), order.data_ptr(),
                                  wtop.data_ptr(), stream)
    assert rc == 0, dm.last_error()


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("T", [100, 301, 1030])
def test_pinned_pageable_device_identical(port, name, T):
    layer = synth.make_layer(**LAYERS[name])
    Xh = synth.make_tokens(layer, T, 700 + T)
    L = dm.lib()
    keep: list = []
    desc = dm.layer_desc(layer, keep)
    H, K = layer.hidden, layer.n_used
    res = {}
    # page-locked host buffers (twice: the second call replays the captured host graph)
    Xp = torch.from_numpy(Xh).pin_memory()
    for rep in range(2):
        outs = (torch.empty((T, H)).pin_memory(), torch.empty((T, K), dtype=torch.int32).pin_memory(),
                torch.empty((T, K)).pin_memory())
        call(L, desc, Xp, T, *outs)
        res[f"pinned{rep}"] = [o.numpy().copy() for o in outs]
    # pageable host buffers
    outs = (torch.empty((T, H)), torch.empty((T, K), dtype=torch.int32), torch.empty((T, K)))
    call(L, desc, torch.from_numpy(Xh.copy()), T, *outs)
    res["pageable"] = [o.numpy().copy() for o in outs]
    # device buffers on a stream
    dev = torch.device("cuda")
    s = torch.cuda.Stream()
    outs = (torch.empty((T, H), device=dev), torch.empty((T, K), dtype=torch.int32, device=dev),
            torch.empty((T, K), device=dev))
    Xd = torch.from_numpy(Xh).to(dev)
    torch.cuda.synchronize()
    call(L, desc, Xd, T, *outs, stream=ct.c_void_p(s.cuda_stream))
    s.synchronize()
    res["device"] = [o.cpu().numpy() for o in outs]
    for k in ("pinned0", "pinned1", "pageable"):
        for a, b in zip(res[k], res["device"]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), k
    out, order, wtop = res["pinned0"]
    o_ref, w_ref = port.route(layer, Xh)
    assert np.array_equal(order, o_ref)
    assert np.array_equal(wtop.view(np.uint32), w_ref.view(np.uint32))
    assert rel_l2(out, port.layer_forward(layer, Xh)) <= 1e-3
