"""Expert parallelism on CPU: the exchange logic of dracomancer_llmengine_b200.ep with the host
restatement of each rank's work (tests/ep_host_ops.py), in one process (emulated exchange) and
over a two-rank gloo process group.  The reference is the single-process layer of the oracle."""
import os
import socket
import types

import numpy as np
import pytest
import torch

from dracomancer_llmengine_b200 import synth
from dracomancer_llmengine_b200.ep import ExpertParallelMoE, emulate
from ep_host_ops import HostOps, plan_ref

LAYERS = {
    "softmax_shared": dict(hidden=256, n_exp=8, n_used=2, inter=256, shared_inter=256, seed=31),
    "sigmoid_bias": dict(hidden=256, n_exp=16, n_used=4, inter=256, scoring="sigmoid", w_scale=2.5, bias=True,
                         seed=32),
}


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_plan_ref_layout():
    order = np.array([[0, 5], [6, 7], [1, 2], [-1, 3]], np.int32)   # E=8 over G=2: rank0 0-3, rank1 4-7
    counts, row_of, src = plan_ref(order, 8, 2, 0)
    assert counts.tolist() == [3, 2]
    assert row_of.tolist() == [[0, 3], [-1, 4], [1, -1], [2, -1]]
    assert src[:5].tolist() == [0, 2, 3, 0, 1]
    counts, row_of, src = plan_ref(order, 8, 2, 4)
    assert row_of.tolist() == [[0, 4], [-1, 5], [1, -1], [2, -1]]
    assert src[[0, 1, 2, 4, 5]].tolist() == [0, 2, 3, 0, 1]


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("G,exchange,Ts", [(1, "fixed", [5]), (2, "fixed", [5, 3]), (2, "compact", [5, 3]),
                                           (4, "compact", [5, 3, 6, 4]), (4, "fixed", [5, 0, 6, 4]),
                                           (4, "compact", [0, 3, 0, 4])])
def test_emulated_ranks_match_single_process(port, name, G, exchange, Ts):
    """Ranks with ragged token counts, including ranks without tokens, in one process."""
    layer = synth.make_layer(**LAYERS[name])
    if layer.n_exp // G < layer.n_used:
        pytest.skip("fewer experts per rank than n_used")
    xs = [synth.make_tokens(layer, T, 100 + i, False) for i, T in enumerate(Ts)]
    ranks = [ExpertParallelMoE(layer, max(Ts), comm=types.SimpleNamespace(world=G, rank=r),
                               ops=HostOps(layer, r, G, port), exchange=exchange) for r in range(G)]
    outs = emulate(ranks, [torch.from_numpy(x) for x in xs])
    ref = port.layer_forward(layer, np.concatenate(xs))
    got = np.concatenate([o.numpy() for o in outs])
    if G == 1:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert rel(got, ref) < 1e-6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port_no, name, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Port
        port = Port()
        layer = synth.make_layer(**LAYERS[name])
        Ts = [5, 3]
        xs = [synth.make_tokens(layer, T, 100 + i, False) for i, T in enumerate(Ts)]
        res = {}
        for exchange in ("fixed", "compact"):
            ep = ExpertParallelMoE(layer, max(Ts), ops=HostOps(layer, rank, world, port), exchange=exchange)
            res[exchange] = ep.forward(torch.from_numpy(xs[rank])).numpy().copy()
            res[exchange + "_again"] = ep.forward(torch.from_numpy(xs[rank])).numpy().copy()
        allx = torch.from_numpy(np.concatenate(xs))
        rep = ExpertParallelMoE(layer, allx.shape[0], ops=HostOps(layer, rank, world, port), layout="replicated")
        res["replicated"] = rep.forward(allx).numpy().copy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", list(LAYERS))
def test_gloo_two_ranks(port, tmp_path, name):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_gloo_worker, args=(world, _free_port(), name, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    layer = synth.make_layer(**LAYERS[name])
    xs = [synth.make_tokens(layer, T, 100 + i, False) for i, T in enumerate([5, 3])]
    ref = port.layer_forward(layer, np.concatenate(xs))
    r = [np.load(os.path.join(tmp_path, f"rank{i}.npz")) for i in range(world)]
    for exchange in ("fixed", "compact"):
        got = np.concatenate([r[0][exchange], r[1][exchange]])
        assert rel(got, ref) < 1e-6, exchange
        again = np.concatenate([r[0][exchange + "_again"], r[1][exchange + "_again"]])
        assert np.array_equal(got, again), "repeat call differs"
    assert np.array_equal(r[0]["fixed"], r[0]["compact"])
    assert rel(r[0]["replicated"], ref) < 1e-6
    assert np.array_equal(r[0]["replicated"], r[1]["replicated"])
