"""Expert parallelism on the GPU: the exchange kernels (plan, pack, combine) bit-exact against
the host restatement, the routed-experts entry point on expert slices, the whole expert-parallel
layer with G ranks emulated on one GPU, and (with two or more GPUs) over NCCL."""
import ctypes as ct
import os
import socket
import types

import numpy as np
import pytest
import torch

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth
from dracomancer_llmengine_b200.ep import DeviceOps, ExpertParallelMoE, PeerBuffers, emulate, slice_desc
from ep_host_ops import plan_ref

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("T,E,K,G,pad", [(1, 8, 2, 2, 0), (300, 128, 8, 8, 0), (300, 128, 8, 8, 7),
                                         (2500, 384, 8, 8, 0), (2500, 384, 8, 16, 3), (77, 60, 6, 3, 0),
                                         (64, 256, 8, 1, 0), (40, 64, 4, 4, 40)])
def test_exchange_kernels_match_host(dlib, T, E, K, G, pad):
    rng = np.random.default_rng(T * 31 + G)
    order = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    order[rng.random((T, K)) < 0.05] = -1          # dropped entries
    order[rng.random((T, K)) < 0.02] = E + 3       # out of range: skipped
    wtop = rng.random((T, K), dtype=np.float32)
    H = 256
    x = rng.standard_normal((T, H), dtype=np.float32)
    block = T + pad if pad else 0
    counts, row_of, src = plan_ref(order, E, G, block)
    cap = G * block if block else T * min(K, G)
    dev = torch.device("cuda")
    d_order, d_w, d_x = (torch.from_numpy(a).to(dev) for a in (order, wtop, x))
    d_counts = torch.full((G,), -7, dtype=torch.int32, device=dev)
    d_row = torch.full((T, G), -7, dtype=torch.int32, device=dev)
    d_src = torch.full((max(cap, 1),), -7, dtype=torch.int32, device=dev)
    assert dlib.draco_b200_ep_plan(d_order.data_ptr(), T, K, E, G, block, d_counts.data_ptr(), d_row.data_ptr(),
                                   d_src.data_ptr(), _s()) == 0, dm.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(d_counts.cpu().numpy(), counts)
    assert np.array_equal(d_row.cpu().numpy(), row_of)
    valid = src >= 0
    assert np.array_equal(d_src.cpu().numpy()[valid], src[valid])

    send_x = torch.full((cap, H), 5.0, device=dev)
    send_m = torch.full((cap, 2 * K), -9, dtype=torch.int32, device=dev)
    assert dlib.draco_b200_ep_pack(d_x.data_ptr(), d_order.data_ptr(), d_w.data_ptr(), d_counts.data_ptr(), G,
                                   d_src.data_ptr(), block, cap, K, H, send_x.data_ptr(), send_m.data_ptr(),
                                   _s()) == 0, dm.last_error()
    torch.cuda.synchronize()
    sx, sm = send_x.cpu().numpy(), send_m.cpu().numpy()
    rows = np.nonzero(valid)[0]
    assert np.array_equal(sx[rows], x[src[rows]])
    assert np.array_equal(sm[rows, :K], order[src[rows]])
    assert np.array_equal(sm[rows, K:].view(np.float32), wtop[src[rows]])
    if block:
        pad_rows = np.array([r for r in range(cap) if not valid[r]], np.int64)
        if pad_rows.size:
            assert (sm[pad_rows, :K] == -1).all() and (sm[pad_rows, K:] == 0).all()

    back = rng.standard_normal((max(cap, 1), H), dtype=np.float32)
    sh = rng.standard_normal((T, H), dtype=np.float32)
    d_back, d_sh = torch.from_numpy(back).to(dev), torch.from_numpy(sh).to(dev)
    out = torch.empty((T, H), device=dev)
    for use_sh in (False, True):
        assert dlib.draco_b200_ep_combine(d_back.data_ptr(), d_row.data_ptr(), T, G, H,
                                          d_sh.data_ptr() if use_sh else None, out.data_ptr(), _s()) == 0
        torch.cuda.synchronize()
        acc = np.zeros((T, H), np.float32)
        for r in range(G):
            m = row_of[:, r] >= 0
            acc[m] += back[row_of[m, r]]
        if use_sh:
            acc += sh
        assert np.array_equal(out.cpu().numpy().view(np.uint32), acc.view(np.uint32))


LAYERS = {
    "softmax_e64_shared": dict(hidden=2048, n_exp=64, n_used=8, inter=512, shared_inter=512, seed=41),
    "sigmoid_groups_e128": dict(hidden=2048, n_exp=128, n_used=8, inter=256, scoring="sigmoid", n_group=8,
                                n_group_used=4, w_scale=2.5, bias=True, shared_inter=256, seed=42),
}


def test_ep_hot_experts_p2p_emulated(port):
    """Zipf-skewed routing (a few experts take most tokens, so one owner gets far more rows than the
    others) through the peer-memory exchange of 4 ranks on one GPU."""
    layer = synth.make_layer(hidden=1024, n_exp=64, n_used=8, inter=512, scoring="sigmoid", w_scale=2.0,
                             bias=True, zipf=True, shared_inter=256, seed=44)
    G, T = 4, 120
    xs = [synth.make_tokens(layer, T, 500 + i, zipf=True) for i in range(G)]
    dev = torch.device("cuda")
    order, _ = port.route(layer, np.concatenate(xs))
    per_rank = np.bincount(order.reshape(-1) // (layer.n_exp // G), minlength=G)
    assert per_rank.max() > 1.5 * per_rank.min()      # the skew reaches the owners
    ranks = [ExpertParallelMoE(layer, T, comm=types.SimpleNamespace(world=G, rank=r),
                               ops=DeviceOps(layer, r, G, dev), exchange="p2p") for r in range(G)]
    outs = emulate(ranks, [torch.from_numpy(x).to(dev) for x in xs])
    torch.cuda.synchronize()
    got = np.concatenate([o.cpu().numpy() for o in outs])
    for r in ranks:
        r.close()
    assert rel(got, port.layer_forward(layer, np.concatenate(xs))) < REL_L2_TOL


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("T", [3, 200])
def test_experts_forward_given_routing(dlib, port, name, T):
    layer = synth.make_layer(**LAYERS[name])
    X = synth.make_tokens(layer, T, 5, False)
    keep: list = []
    full = dm.layer_desc(layer, keep)
    K = layer.n_used
    ref_out = dm.forward(layer, X)
    order, wtop = dm.route(layer, X)
    # whole expert set, routing given, shared on: the same output as the routed call
    out = np.empty_like(ref_out)
    assert dlib.draco_b200_experts_forward(ct.byref(full), X.ctypes.data, T, order.ctypes.data, wtop.ctypes.data,
                                           0, 0, out.ctypes.data, 1, 0, None) == 0, dm.last_error()
    assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32))
    # routing rows with a stride (device buffers, asynchronous), summed over four expert slices
    dev = torch.device("cuda")
    meta = np.zeros((T, 2 * K), np.int32)
    meta[:, :K] = order
    meta[:, K:] = wtop.view(np.int32)
    d_meta, d_x = torch.from_numpy(meta).to(dev), torch.from_numpy(X).to(dev)
    G = 4
    e_loc = layer.n_exp // G
    total = np.zeros_like(ref_out)
    for r in range(G):
        d = slice_desc(full, r * e_loc, e_loc, keep)
        part = torch.empty((T, layer.hidden), device=dev)
        assert dlib.draco_b200_experts_forward(ct.byref(d), d_x.data_ptr(), T, d_meta.data_ptr(),
                                               d_meta.data_ptr() + 4 * K, 2 * K, r * e_loc, part.data_ptr(), 0, 0,
                                               _s()) == 0, dm.last_error()
        total += part.cpu().numpy()
    sh = torch.empty((T, layer.hidden), device=dev)
    assert dlib.draco_b200_experts_forward(ct.byref(full), d_x.data_ptr(), T, None, None, 0, 0, sh.data_ptr(), 1, 0,
                                           _s()) == 0, dm.last_error()
    # fp16 activation rows give the same bits as fp32 rows holding the same values: the
    # tensor-core path (T = 200) reads them as they are, the CUDA-core path (T = 3) widens them
    d_meta_o, d_meta_w = d_meta.data_ptr(), d_meta.data_ptr() + 4 * K
    o32 = torch.empty((T, layer.hidden), device=dev)
    o16 = torch.empty((T, layer.hidden), device=dev)
    x16 = d_x.half()
    for xx, oo, flag in ((d_x.half().float(), o32, 0), (x16, o16, 1)):
        assert dlib.draco_b200_experts_forward(ct.byref(full), xx.data_ptr(), T, d_meta_o, d_meta_w, 2 * K, 0,
                                               oo.data_ptr(), 1, flag, _s()) == 0, dm.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(o16.cpu().numpy().view(np.uint32), o32.cpu().numpy().view(np.uint32))
    sh_h = sh.cpu().numpy()
    sh_ref = port.shared_add(layer, X, np.zeros_like(ref_out))
    assert rel(sh_h, sh_ref) < REL_L2_TOL
    total += sh_h
    # a slice holds fewer experts, so its token tiles (and the MMA shapes) can differ from the
    # whole-set call's: agreement to a few fp32 ulps of the fp16-operand products
    assert rel(total, ref_out) < 1e-4
    assert rel(total, port.layer_forward(layer, X)) < REL_L2_TOL


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("G,exchange,T", [(2, "fixed", 40), (4, "compact", 150), (8, "fixed", 96),
                                          (8, "compact", 5)])
def test_ep_emulated_on_one_gpu(port, name, G, exchange, T):
    layer = synth.make_layer(**LAYERS[name])
    Ts = [T - (i % 3) for i in range(G)]
    xs = [synth.make_tokens(layer, t, 200 + i, False) for i, t in enumerate(Ts)]
    dev = torch.device("cuda")
    ranks = [ExpertParallelMoE(layer, max(Ts), comm=types.SimpleNamespace(world=G, rank=r),
                               ops=DeviceOps(layer, r, G, dev), exchange=exchange) for r in range(G)]
    outs = emulate(ranks, [torch.from_numpy(x).to(dev) for x in xs])
    torch.cuda.synchronize()
    got = np.concatenate([o.cpu().numpy() for o in outs])
    X = np.concatenate(xs)
    assert rel(got, port.layer_forward(layer, X)) < REL_L2_TOL
    # same layer on one GPU, in per-rank token batches: the path choice may differ, the result
    # agrees to fp16-operand rounding
    single = np.concatenate([dm.forward(layer, x) for x in xs])
    assert rel(got, single) < 2 * REL_L2_TOL


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("G,T", [(2, 40), (4, 150), (8, 96), (4, 0)])
def test_ep_p2p_emulated_matches_fixed_exchange(port, name, G, T):
    """Peer-memory dispatch/combine on G ranks sharing one GPU, with the owners storing their
    results into the homes' buffers (push) or the homes loading them (pull): the same rows reach
    the owners as with the fixed-block all-to-all, so the outputs are identical.  T = 0: every
    other rank has no tokens."""
    layer = synth.make_layer(**LAYERS[name])
    Ts = [T - (i % 3) for i in range(G)] if T else [(23 if i % 2 else 0) for i in range(G)]
    xs = [torch.from_numpy(synth.make_tokens(layer, t, 400 + i, False)).cuda() for i, t in enumerate(Ts)]
    dev = torch.device("cuda")
    res = {}
    for exchange, results in (("fixed", "push"), ("p2p", "push"), ("p2p", "pull")):
        ranks = [ExpertParallelMoE(layer, max(Ts), comm=types.SimpleNamespace(world=G, rank=r),
                                   ops=DeviceOps(layer, r, G, dev), exchange=exchange, results=results)
                 for r in range(G)]
        outs = emulate(ranks, xs)
        torch.cuda.synchronize()
        res[exchange if exchange == "fixed" else results] = np.concatenate([o.cpu().numpy() for o in outs])
        for r in ranks:
            r.close()
    assert np.array_equal(res["push"].view(np.uint32), res["fixed"].view(np.uint32))
    assert np.array_equal(res["pull"].view(np.uint32), res["fixed"].view(np.uint32))
    res["p2p"] = res["push"]
    X = np.concatenate([x.cpu().numpy() for x in xs])
    assert rel(res["p2p"], port.layer_forward(layer, X)) < REL_L2_TOL


def test_ep_p2p_graph_replay_matches_eager(port):
    """The whole peer-memory step (routing, plan, push, barriers, routed experts, shared expert,
    pull) captured in one CUDA graph gives the eager step's bits, also after new inputs."""
    layer = synth.make_layer(**LAYERS["softmax_e64_shared"])
    dev = torch.device("cuda")
    T = 64
    ep = ExpertParallelMoE(layer, T, comm=types.SimpleNamespace(world=1, rank=0), ops=DeviceOps(layer, 0, 1, dev),
                           exchange="p2p")
    x = torch.from_numpy(synth.make_tokens(layer, T, 600, False)).to(dev)
    out = torch.empty((T, layer.hidden), device=dev)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        g = ep.capture(x, out)
        assert ep.launches_per_step >= 8   # route, plan, push, barriers, expert GEMMs, pull
        for seed in (601, 602):
            x.copy_(torch.from_numpy(synth.make_tokens(layer, T, seed, False)))
            g.replay()
            got = out.clone()
            want = ep.forward(x, torch.empty_like(out)).clone()
    torch.cuda.synchronize()
    ep.check()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32))
    assert rel(want.cpu().numpy(), port.layer_forward(layer, x.cpu().numpy())) < REL_L2_TOL
    del g
    ep.close()


def test_ep_barrier_one_rank_and_bounded_wait(dlib):
    """The flag barrier: alone it passes at once and counts epochs; with a second rank that never
    arrives (a flag nothing sets) it gives up after its time limit, reports 0x400 and the device
    stays usable."""
    import time
    dev = torch.device("cuda")
    pb = PeerBuffers(1, 0, 1, 4, 1, dev)
    pb.link([dict(pb.own)])
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        assert dlib.draco_b200_ep_barrier(pb.peer_flags.data_ptr(), pb.my_flags, pb.epoch, 1, 0, pb.status, s) == 0
    torch.cuda.synchronize()
    from dracomancer_llmengine_b200.ep import tensor_at
    ctl = tensor_at(pb.own["ctl"], (64,), torch.int32, dev).cpu().numpy()
    assert ctl[0] == 3 and ctl[16] == 3 and ctl[32] == 0      # flag, epoch, status
    # two ranks, the second absent
    other = PeerBuffers(1, 0, 1, 4, 1, dev)
    pb2 = PeerBuffers(2, 0, 1, 4, 1, dev)
    pb2.link([dict(pb2.own), dict(other.own)])
    t0 = time.time()
    assert dlib.draco_b200_ep_barrier(pb2.peer_flags.data_ptr(), pb2.my_flags, pb2.epoch, 2, 0, pb2.status, s) == 0
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert int(pb2.status_t.item()) == 0x400
    assert 1.0 < waited < 30.0
    assert torch.ones(4, device=dev).sum().item() == 4.0
    for b in (pb, other, pb2):
        b.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port_no, name, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        layer = synth.make_layer(**LAYERS[name])
        Ts = [64 + 9 * i for i in range(world)]
        xs = [synth.make_tokens(layer, t, 300 + i, False) for i, t in enumerate(Ts)]
        res = {}
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            for exchange in ("fixed", "compact", "p2p", "p2p_pull"):
                ep = ExpertParallelMoE(layer, max(Ts), exchange=exchange.split("_")[0], device=dev,
                                       results="pull" if exchange.endswith("pull") else "push")
                x = torch.from_numpy(xs[rank]).to(dev)
                res[exchange] = ep.forward(x).cpu().numpy()
                res[exchange + "_again"] = ep.forward(x).cpu().numpy()
                ep.check()
                ep.close()
            allx = torch.from_numpy(np.concatenate(xs)).to(dev)
            rep = ExpertParallelMoE(layer, allx.shape[0], layout="replicated", device=dev)
            res["replicated"] = rep.forward(allx).cpu().numpy()
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", list(LAYERS))
def test_ep_nccl(port, tmp_path, name):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    mp.start_processes(_nccl_worker, args=(world, _free_port(), name, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    layer = synth.make_layer(**LAYERS[name])
    xs = [synth.make_tokens(layer, 64 + 9 * i, 300 + i, False) for i in range(world)]
    X = np.concatenate(xs)
    ref = port.layer_forward(layer, X)
    r = [np.load(os.path.join(tmp_path, f"rank{i}.npz")) for i in range(world)]
    for exchange in ("fixed", "compact", "p2p", "p2p_pull"):
        got = np.concatenate([r[i][exchange] for i in range(world)])
        assert rel(got, ref) < REL_L2_TOL, exchange
        again = np.concatenate([r[i][exchange + "_again"] for i in range(world)])
        assert np.array_equal(got, again)
    for i in range(world):
        assert np.array_equal(r[i]["fixed"], r[i]["compact"])
        assert np.array_equal(r[i]["fixed"], r[i]["p2p"])
        assert np.array_equal(r[i]["fixed"], r[i]["p2p_pull"])
        assert np.array_equal(r[i]["replicated"], r[0]["replicated"])
    assert rel(r[0]["replicated"], ref) < REL_L2_TOL
