"""Benchmark of the MoE FFN layer (metric: MoE layer tok/s, with HBM GB/s and TFLOP/s against the
B200 roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--configs A,B|none]
                    [--impl draco|reference]

One step = one MoE layer forward (routing, grouped expert gate/up/down, combine, shared expert
when the layer has one) over a configuration's token batch, synthetic seeded weights and
activations (dracomancer_llmengine_b200.synth).  The headline (the line's top-level keys) is the
second benchmark configuration, chunked prefill of 512 tokens through the H2048/E128/top-8/F768
Q4_K+Q6_K layer; `configs` in the same line holds one record per other configuration (decode
cfg1, K2 decode cfg3, Ling prefill cfg4, Zipf K2 prefill cfg5), each with its own throughput,
roofline, parity check and CPU baseline.

  value  device-resident throughput: inputs already in HBM, CUDA events on the launching
         stream (a dedicated non-default stream); weights and activations larger than L2 (the
         cfg1 decode weights are evicted by a 256 MB write and read between steps).  Phase
         times (and the dominant kernel's, for the roofline) come from a second pass of the same
         steps with the library's per-phase events on.
  e2e    the same layer through the C ABI with pinned host X/out: the host->device copy of X and
         the device->host copy of the output are inside the timed region.
  parity outside the timed region: the timed call's routing (every token) against the C
         restatement of the reference routers (bit-exact) and its output against the
         reference's own m6_moe_tok (oracle/_ref) + shared expert, rel-L2.

Under torchrun (N > 1) the layer runs expert-parallel (dracomancer_llmengine_b200.ep): each rank
holds E/N experts.  Headline: each rank has its own 512 tokens (weak scaling), routes them,
stores token rows into the expert owners' receive buffers over NVLink (peer memory, one CUDA
graph per step), and adds the owners' partial rows and the shared expert at home.  Records:
cfg3 in the replicated decode layout (every rank routes the same 64 tokens, an all-reduce sums
the partial outputs), cfg4/cfg5 with the configuration's batch split over the ranks (strong
scaling).  Times are the max over ranks; `value` counts the tokens of all ranks.  Parity at
N > 1: rank 0 gathers sampled output rows, every rank computes the oracle's partial sums of
those rows over its own expert slice, and rank 0 adds them.

`--impl reference` times the reference's own CPU path of the layer on the host cores with every
host thread: routing restated from src/qwen35_prefill.py:180-188 (numpy) + the reference's
m6_moe_tok with its fused AVX-512 GEMM (oracle/_ref, compiled from the reference's sources);
rank 0 only.
"""
from __future__ import annotations

import os
import sys

# the reference arm runs on every host core, also under torchrun (which exports
# OMP_NUM_THREADS=1): set the thread counts before numpy/OpenBLAS and libgomp read them
if any(a == "reference" or a == "--impl=reference" for a in sys.argv) and \
        os.environ.get("RANK", "0") == "0":
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = str(os.cpu_count() or 1)

import argparse  # noqa: E402
import dataclasses  # noqa: E402
import json  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import tempfile  # noqa: E402
import time  # noqa: E402

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tok/s + HBM GB/s vs 8 TB/s (decode), TFLOP/s (prefill), 1-8 GPU"
DTYPE = "fp16 operands (weights dequantised from Q4_K/Q6_K, activations), fp32 accumulate"
SUB_CONFIGS = ("cfg1_decode", "cfg3_k2_decode", "cfg4_ling_prefill", "cfg5_k2_prefill_zipf")
DECODE = ("cfg1_decode", "cfg3_k2_decode")
REL_L2_TOL = 1e-3


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def layer_work(layer, order, T, experts=None):
    """Algorithmic bytes and FLOPs of one layer call (weights of distinct experts touched once,
    router, activations in/out), and the gate/up kernel's share.  `experts` = (first, count)
    restricts the expert work to one rank's slice (expert parallelism; `order` then holds the
    routing of every rank's tokens)."""
    from dracomancer_llmengine_b200.synth import row_bytes
    H, F = layer.hidden, layer.inter
    lo, n = experts if experts else (0, layer.n_exp)
    order = np.where((order >= lo) & (order < lo + n), order, -1)
    distinct = len(np.unique(order[(order >= 0) & (order < layer.n_exp)]))
    gu = 2 * F * row_bytes(layer.code_gu, H)
    dn = H * row_bytes(layer.code_d, F)
    sh = 0
    if layer.shared_inter:
        sh = 2 * layer.shared_inter * row_bytes(layer.code_gu, H) + H * row_bytes(layer.code_d, layer.shared_inter)
    router = layer.n_exp * H * 4
    io = 2 * T * H * 4
    total_bytes = distinct * (gu + dn) + sh + router + io
    assign = int(((order >= 0) & (order < layer.n_exp)).sum())
    flops = 2 * 3 * H * F * assign + (2 * 3 * H * layer.shared_inter * T if layer.shared_inter else 0) \
        + 2 * T * layer.n_exp * H
    # the gate/up grouped GEMM kernel: gate+up weights of the distinct experts, the fp16 token
    # row of every assignment in, the fp16 SwiGLU activation of every assignment out
    gateup_bytes = distinct * gu + assign * H * 2 + assign * F * 2
    return dict(distinct=distinct, bytes=total_bytes, flops=flops, gateup_bytes=gateup_bytes,
                gateup_flops=2 * 2 * H * F * assign, assignments=assign)


def profiled_traffic(config: str, kernel: str = "tc_gemm", algorithmic_bytes: float = 0.0):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary of this
    workload (profiles/<kernel>_<config>.md): the line `traffic_bytes_per_launch: N` of a
    capture at full size, or `traffic_per_algorithmic_byte: r` of a capture on a smaller case of
    the same kernel, scaled here by this launch's algorithmic bytes; else None."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        try:
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
            if line.startswith("traffic_per_algorithmic_byte:") and algorithmic_bytes:
                return int(float(line.split(":", 1)[1].strip()) * algorithmic_bytes)
        except ValueError:
            return None
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        # nvidia-smi takes a while to start (driver library initialisation): the timed region
        # starts only after its first sample is written
        t0 = time.perf_counter()
        while self.proc and time.perf_counter() - t0 < 10.0 and os.path.getsize(self.path) == 0:
            time.sleep(0.02)
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------- reference CPU path
def numpy_route(layer, X):
    """The drivers' numpy routers: softmax top-k renorm with the clamp (src/qwen35_prefill.py:
    180-188), sigmoid + bias selection, weights renormalised and scaled (src/k2_prefill.py:
    122-127)."""
    K = layer.n_used
    lg = X @ np.ascontiguousarray(layer.gate_inp).T
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
        w = w / w.sum(1, keepdims=True)
        if layer.w_scale not in (0.0, 1.0):
            w = w * layer.w_scale
    return np.ascontiguousarray(order, np.int32), np.ascontiguousarray(w, np.float32)


def cpu_reference(layer, X, steps, warmup, budget_s=None):
    """The reference's CPU path on the host cores: numpy routing as the drivers do it, then the
    reference's own m6_moe_tok and (when the layer has one) its shared expert through the same
    entry point; the restatement (oracle/libmoe_oracle.so) where the reference's C is not built."""
    from oracle.oracle import Ref, Port, ref_available
    if ref_available():
        R, kind = Ref(), "reference"
    else:
        R, kind = Port(), "port"

    def step():
        order, w = numpy_route(layer, X)
        out = R.moe_tok(layer, X, order, w)
        if layer.shared_inter:
            R.shared_add(layer, X, out)
        return out

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    for i in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if budget_s and time.perf_counter() - t_start > budget_s and i >= 1:
            break
    return kind, times


def cpu_baseline_record(name, layer, X, budget_s):
    """Bounded sample of the reference CPU path on this workload (rank 0, N = 1)."""
    from oracle.oracle import Ref, ref_available
    T = X.shape[0]
    if name == "cfg1_decode" and ref_available():
        # the decode entry point of the reference, one token per call (src/m6_layer.c:771-802)
        R = Ref()
        R.decode(layer, X[:1])
        times = []
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < budget_s and len(times) < 200:
            t1 = time.perf_counter()
            R.decode(layer, X[:1])
            times.append(time.perf_counter() - t1)
        ms = statistics.median(times) * 1e3
        return {"value": 1 / (ms / 1e3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"{len(times)} single-token m6_granite_moe calls (scalar kernels), median"}
    n = T
    if T * layer.hidden * layer.inter > 512 * 7168 * 2048:   # cfg5: a 512-token slice of the batch
        n = 512
    kind, times = cpu_reference(layer, X[:n], steps=100, warmup=1, budget_s=budget_s)
    ms = statistics.median(times) * 1e3
    return {"value": n / (ms / 1e3), "unit": "tok/s", "cores": os.cpu_count(), "kind": kind,
            "sample": f"{len(times)} layer calls of {n} of the workload's {T} tokens (numpy routing + "
                      f"m6_moe_tok + shared expert), median"}


# ------------------------------------------------------------------------- parity
def local_view(layer):
    """The layer's expert slice as a layer of its own (expert ids 0 .. count-1)."""
    n = layer.gate.shape[0]
    return dataclasses.replace(layer, n_exp=n, expert0=0)


def parity_check(layer, Xs, outs, orders, wtops, sample, world, rank, comm, experts, replicas=False):
    """Routing of every token (all ranks' batches) bit-exact against the C restatement of the
    reference routers; output rows of a seeded sample against the reference's m6_moe_tok (+
    shared expert).  At N > 1 every rank computes the oracle's partial sums of the sampled rows
    over its own expert slice (the slice it holds on the host) and rank 0 adds them; with
    `replicas` (every rank runs the whole layer on its own tokens) rank 0 checks all ranks' rows
    against the whole layer.  Xs, outs, orders, wtops: this rank's arrays.  Returns the record on
    rank 0."""
    from oracle.oracle import Port, Ref, ref_available
    port = Port()
    T = Xs.shape[0]
    routing_ok = True
    n_routed = 0
    if T:
        o_ref, w_ref = port.route(layer, Xs)
        routing_ok = bool(np.array_equal(o_ref, orders) and
                          np.array_equal(w_ref.view(np.uint32), np.ascontiguousarray(wtops).view(np.uint32)))
        n_routed = T
    rng = np.random.default_rng(777 + rank)
    rows = np.sort(rng.choice(T, size=min(sample, T), replace=False)) if T else np.zeros(0, np.int64)
    mine = (Xs[rows], orders[rows], wtops[rows], outs[rows])
    allv = comm.all_gather_object(mine) if world > 1 else [mine]
    ok_all = comm.all_gather_object(routing_ok) if world > 1 else [routing_ok]
    nr_all = comm.all_gather_object(n_routed) if world > 1 else [n_routed]
    X_s = np.concatenate([a[0] for a in allv])
    o_s = np.concatenate([a[1] for a in allv])
    w_s = np.concatenate([a[2] for a in allv])
    got = np.concatenate([a[3] for a in allv])
    R = Ref() if ref_available() else port
    lo, cnt = experts if experts else (0, layer.n_exp)
    o_loc = np.where((o_s >= lo) & (o_s < lo + cnt), o_s - lo, -1).astype(np.int32)
    part = R.moe_tok(local_view(layer) if experts else layer, X_s, o_loc, w_s) if len(X_s) else np.zeros((0, layer.hidden), np.float32)
    parts = comm.all_gather_object(part) if world > 1 and not replicas else [part]
    if rank:
        return None
    want = np.sum(np.stack([p.astype(np.float64) for p in parts]), axis=0).astype(np.float32)
    if layer.shared_inter and len(X_s):
        (R if hasattr(R, "shared_add") else port).shared_add(layer, X_s, want)
    err = float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want.astype(np.float64)), 1e-30))
    return {"routing_bitexact": bool(all(ok_all)), "tokens_routing_checked": int(sum(nr_all)),
            "rel_l2": err, "rel_l2_tol": REL_L2_TOL, "tokens_output_checked": int(len(X_s)),
            "pass": bool(all(ok_all) and err <= REL_L2_TOL),
            "oracle": "routing: C restatement of src/m6_layer.c routers (pinned to the reference); output: "
                      + ("reference m6_moe_tok (oracle/_ref)" if ref_available() else "C restatement")}


class SoloComm:
    def all_gather_object(self, obj):
        return [obj]


class DistComm:
    def __init__(self, dist):
        self.dist = dist

    def all_gather_object(self, obj):
        out = [None] * self.dist.get_world_size()
        self.dist.all_gather_object(out, obj)
        return out


# ------------------------------------------------------------------------- one workload
def run_workload(name, args, ctx, headline):
    """Time one configuration on this process's GPU (expert-parallel over the group at N > 1);
    returns the record (rank 0) or None."""
    import ctypes as ct
    import torch
    import dracomancer_llmengine_b200 as dm
    from dracomancer_llmengine_b200 import synth
    world, rank, local, dist, dev = ctx["world"], ctx["rank"], ctx["local"], ctx["dist"], ctx["dev"]
    L = dm.lib()
    cfgd = synth.CONFIGS[name]
    T_cfg = cfgd["tokens"]
    layout, scaling = "a2a", "weak"
    if world > 1 and not headline:
        if name == "cfg1_decode":
            # one decode token does not shard: sharding its 8 experts over GPUs only adds an
            # exchange to a 50 us layer, so every GPU runs the whole layer on its own token
            layout, scaling = "replicas", "weak"
        elif name in DECODE:
            layout, scaling = "replicated", "strong"
        else:
            scaling = "strong"
    T = T_cfg if (world == 1 or headline or layout in ("replicated", "replicas")) else T_cfg // world
    t_gen = time.perf_counter()
    experts = (rank * (cfgd["n_exp"] // world), cfgd["n_exp"] // world) if world > 1 and layout != "replicas" else None
    layer, Xfull = synth.make_config(name, experts=experts)
    if world > 1 and (headline or layout == "replicas") and rank:
        Xh = synth.make_tokens(layer, T, cfgd["seed"] + 1000 * rank, cfgd["zipf"])
    elif world > 1 and scaling == "strong" and layout == "a2a":
        Xh = np.ascontiguousarray(Xfull[rank * T:(rank + 1) * T])
    else:
        Xh = Xfull
    gen_s = time.perf_counter() - t_gen
    keep: list = []
    desc = dm.layer_desc(layer, keep) if (world == 1 or layout == "replicas") else None
    X = torch.from_numpy(Xh).to(dev)
    out = torch.empty((T, layer.hidden), device=dev, dtype=torch.float32)
    order = torch.empty((T, layer.n_used), device=dev, dtype=torch.int32)
    wtop = torch.empty((T, layer.n_used), device=dev, dtype=torch.float32)
    stream = ctx["stream"]
    ep = None
    if world > 1 and layout != "replicas":
        from dracomancer_llmengine_b200.ep import ExpertParallelMoE
        with torch.cuda.stream(stream):
            ep = ExpertParallelMoE(layer, T, exchange=args.exchange if layout == "a2a" else "fixed",
                                   layout=layout, device=dev)
    graph = None

    def fwd():
        if graph is not None:
            graph.replay()
            return
        if ep is not None:
            ep.forward(X, out)
            return
        rc = L.draco_b200_moe_forward(ct.byref(desc), X.data_ptr(), T, out.data_ptr(), order.data_ptr(),
                                      wtop.data_ptr(), stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(dm.last_error())

    # decode weights of cfg1 fit in L2: between steps write 256 MB (evicts them) and then read
    # another 256 MB, so the dirty lines of the write are written back before the step
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if name == "cfg1_decode" else None
    flush_r = torch.zeros(64 << 20, dtype=torch.float32, device=dev) if flush is not None else None

    def flush_l2():
        flush.zero_()
        flush_r.sum()

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            fwd()
        if ep is not None and layout == "a2a" and args.exchange == "p2p":
            # the expert-parallel step as one CUDA graph (no collective, no host round trip in it)
            try:
                graph = ep.capture(X, out)
                eager = out.clone()           # capture ran one eager step first
                graph.replay()
                stream.synchronize()
                if not torch.equal(out, eager):
                    raise RuntimeError("graph replay differs from the eager step")
            except Exception as exc:   # keep the eager step
                print(f"rank {rank}: graph capture failed ({exc}); timing eager steps", file=sys.stderr)
                graph = None
                torch.cuda.synchronize()
                ep.peer.status_t.zero_()   # the eager steps that follow report their own waits
            for _ in range(2):
                fwd()
    torch.cuda.synchronize()
    if ep is not None:
        my_order = ep._bufs["order"][:T].contiguous()
        my_wtop = ep._bufs["wtop"][:T].contiguous()
        allo = [torch.empty_like(my_order) for _ in range(world)]
        dist.all_gather(allo, my_order)
        order_all = torch.cat(allo).cpu().numpy() if layout == "a2a" else my_order.cpu().numpy()
        wexp = (ep.ops.first, ep.ops.e_loc)
    else:
        my_order, my_wtop = order, wtop
        order_all = order.cpu().numpy()
        wexp = None
    work = layer_work(layer, order_all, T, wexp)

    # ---- value: device-resident timed region ----
    steps = args.steps
    launches0 = L.draco_b200_launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        # the ranks meet after their samplers have started (which takes each a different time),
        # so no rank's first step waits in the exchange for a late one
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            if flush is not None:
                flush_l2()
            ev[i][0].record(stream)
            fwd()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    launches = L.draco_b200_launch_count() - launches0
    if graph is not None:   # replays bypass the host-side counter: the captured step's kernels
        launches = ep.launches_per_step * steps
    step_ms = [a.elapsed_time(b) for a, b in ev]
    # phase times from a second pass with the library's per-phase CUDA events on (eager calls)
    dm.profile(True)
    g_saved, graph = graph, None
    with torch.cuda.stream(stream):
        for i in range(steps):
            if flush is not None:
                flush_l2()
            fwd()
    graph = g_saved
    torch.cuda.synchronize()
    prof = dm.profile_read()
    dm.profile(False)
    tot_ms = float(sum(step_ms))
    if dist:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    ms_per_step = tot_ms / steps
    tokens_step = T if layout == "replicated" else world * T
    value = tokens_step * steps / (tot_ms / 1e3)

    # ---- parity of the last timed call's output (outside the timed region) ----
    with torch.cuda.stream(stream):
        fwd()
    torch.cuda.synchronize()
    comm = DistComm(dist) if dist else SoloComm()
    sample = 512 if (headline and world == 1) else (128 if T <= 1024 else 64)
    if layer.hidden > 4096:
        sample = min(sample, 64)
    parity = parity_check(layer, Xh, out.cpu().numpy(), my_order.cpu().numpy(), my_wtop.cpu().numpy(),
                          sample, world, rank, comm, experts, replicas=layout == "replicas")

    # ---- e2e: through the public API with pinned host buffers ----
    Xp, Op = ctx["pinned"](T, layer.hidden)
    Xp.copy_(torch.from_numpy(Xh))

    def fwd_host():
        if ep is not None:
            with torch.cuda.stream(stream):
                X.copy_(Xp, non_blocking=True)
                fwd()
                Op.copy_(out, non_blocking=True)
            stream.synchronize()
            return
        rc = L.draco_b200_moe_forward(ct.byref(desc), Xp.data_ptr(), T, Op.data_ptr(), None, None, None)
        if rc != 0:
            raise RuntimeError(dm.last_error())

    for _ in range(2):
        fwd_host()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        fwd_host()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = tokens_step * steps / e2e_s

    # ---- roofline of the dominant kernel: the gate/up grouped GEMM, or the fused decode layer ----
    hbm, bf16, src = peaks()
    fused = prof.get("fused", (0.0, 0))[1] > 0
    if fused:   # one kernel does the whole layer: its bytes are the layer's
        gu_ms = prof["fused"][0] / prof["fused"][1]
        kbytes, kflops, kname = work["bytes"], work["flops"], "fused decode layer (routing through combine, one launch)"
    else:
        gu_ms = prof["gateup"][0] / max(prof["gateup"][1], 1)
        kbytes, kflops, kname = work["gateup_bytes"], work["gateup_flops"], "gateup (grouped dequant GEMM, gate+up+SwiGLU)"
    gu_ms = max(gu_ms, 1e-9)
    gu_gbs = kbytes / (gu_ms / 1e3) / 1e9
    gu_tfs = kflops / (gu_ms / 1e3) / 1e12
    tensor_bound = name in ("cfg4_ling_prefill", "cfg5_k2_prefill_zipf")
    roof = {"kernel": kname, "bound": "tensor" if tensor_bound else "hbm",
            "achieved": gu_tfs if tensor_bound else gu_gbs, "peak": bf16 if tensor_bound else hbm,
            "unit": "TFLOP/s" if tensor_bound else "GB/s",
            "frac": (gu_tfs / bf16) if tensor_bound else (gu_gbs / hbm),
            "traffic": (profiled_traffic(name, "fused_decode" if fused else "tc_gemm", kbytes)
                        if world == 1 and not args.overrides else None),
            "algorithmic_bytes": kbytes, "algorithmic_flops": kflops,
            "peak_source": src + (" (cuBLAS bf16 burst; the kernel runs fp16 operands)" if tensor_bound else
                                  " (copy bandwidth)"),
            "kernel_ms": gu_ms, "kernel_gbs": gu_gbs, "kernel_tflops": gu_tfs,
            "layer_gbs": work["bytes"] / (ms_per_step / 1e3) / 1e9,
            "layer_hbm_frac": work["bytes"] / (ms_per_step / 1e3) / 1e9 / hbm,
            "layer_tflops": work["flops"] / (ms_per_step / 1e3) / 1e12,
            "phase_ms": {k: (v[0] / v[1] if v[1] else None) for k, v in prof.items()}}
    par = "single GPU"
    if world > 1:
        par = f"expert parallel x{world}: {layer.n_exp // world} experts/GPU, " + (
            ("peer-memory exchange over NVLink" if args.exchange == "p2p" else f"NCCL all-to-all ({args.exchange})")
            if layout == "a2a" else "replicated tokens, NCCL all-reduce of partial outputs")
        if layout == "replicas":
            par = f"{world} replicas: every GPU runs the whole layer on its own tokens (no exchange)"
    config = {"workload": name, "hidden": cfgd["hidden"], "n_exp": cfgd["n_exp"], "top_k": cfgd["n_used"],
              "ffn": cfgd["inter"], "tokens_per_gpu": T, "tokens_per_step": tokens_step,
              "formats": "Q4_K gate/up, Q6_K down", "shared_ffn": cfgd["shared_inter"], "routing": cfgd["scoring"],
              "l2": "weights and activations exceed L2 (no flush needed)" if name != "cfg1_decode"
              else "decode weights 25 MB fit in L2; flushed between steps by a 256 MB write then a 256 MB read",
              "parallelism": par, "distinct_experts": work["distinct"], "assignments": work["assignments"]}
    if args.overrides:
        config["override"] = dict(args.overrides)
    rec = {"value": value, "unit": "tok/s", "ms_per_step": ms_per_step, "scaling": scaling, "config": config,
           "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": int(T * layer.hidden * 4),
                   "d2h_bytes_per_step": int(T * layer.hidden * 4)},
           "gpu_launches": int(launches), "roofline": roof, "clocks": clk.summary(), "parity": parity,
           "setup_s": {"generate": round(gen_s, 2)}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            rec["cpu_baseline"] = cpu_baseline_record(name, layer, Xh, budget_s=20 if headline else 8)
        except Exception as exc:   # the baseline is reported, never required
            rec["cpu_baseline"] = {"unavailable": str(exc)[:200]}
    if ep is not None:
        ep.check()
        graph = None
        ep.close()
    del X, out, order, wtop, flush, flush_r
    torch.cuda.synchronize()
    L.draco_b200_reset()   # drop this workload's weight copies before the next one
    torch.cuda.empty_cache()
    return rec if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2_prefill", help="the headline workload")
    ap.add_argument("--configs", default=",".join(SUB_CONFIGS),
                    help="comma-separated workloads reported under `configs` ('none': headline only)")
    ap.add_argument("--impl", default="draco", choices=["draco", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--override", default="",
                    help="KEY=VALUE[,KEY=VALUE] changes to the workloads' shape (n_exp, tokens), for profiler "
                         "captures of a smaller case of the same kernels; the line says so in config.override")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "fixed", "compact"],
                    help="expert-parallel token exchange (N > 1): peer-memory stores/loads with flag barriers, "
                         "or NCCL all-to-all with fixed blocks / exchanged counts")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    from dracomancer_llmengine_b200 import synth
    overrides = {}
    for kv in filter(None, args.override.split(",")):
        k, v = kv.split("=", 1)
        if k not in ("n_exp", "tokens"):
            raise SystemExit(f"--override: {k} is not n_exp or tokens")
        overrides[k] = int(v)
    for c in synth.CONFIGS.values():
        c.update(overrides)
    args.overrides = overrides
    cfgd = synth.CONFIGS[args.config]
    T = cfgd["tokens"]

    if args.impl == "reference":
        if rank != 0:
            return
        layer, X = synth.make_config(args.config)
        steps = max(args.steps, 1)
        kind, times = cpu_reference(layer, X, steps, max(args.warmup, 1), budget_s=120)
        ms = statistics.median(times) * 1e3
        v = T / (ms / 1e3)
        cores = os.cpu_count()
        config = {"workload": args.config, "hidden": cfgd["hidden"], "n_exp": cfgd["n_exp"],
                  "top_k": cfgd["n_used"], "ffn": cfgd["inter"], "tokens_per_gpu": T,
                  "formats": "Q4_K gate/up, Q6_K down", "shared_ffn": cfgd["shared_inter"],
                  "routing": cfgd["scoring"]}
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": 0, "steps": len(times),
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF superblocks)",
                "config": config, "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                                 "threads": int(os.environ.get("OMP_NUM_THREADS", cores)),
                                 "sample": f"{len(times)} full layer calls of {T} tokens (median)"},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # page-locked staging buffers for the end-to-end leg, allocated first, as an engine would at
    # start-up (a later allocation of the same size was measured to copy ~1.5x slower); the
    # largest workload's size, sliced per workload
    subs = [c for c in args.configs.split(",") if c and c != "none" and c != args.config]
    for c in subs:
        if c not in synth.CONFIGS:
            raise SystemExit(f"unknown workload {c}")
    sizes = [synth.CONFIGS[c]["tokens"] * synth.CONFIGS[c]["hidden"] for c in [args.config] + subs]
    big = max(sizes)
    Xp_all = torch.empty(big, dtype=torch.float32).pin_memory()
    Op_all = torch.empty(big, dtype=torch.float32).pin_memory()

    def pinned(T_, H_):
        return Xp_all[:T_ * H_].view(T_, H_), Op_all[:T_ * H_].view(T_, H_)

    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    # a dedicated (non-default) stream, as an engine would give the library
    ctx = {"world": world, "rank": rank, "local": local, "dist": dist, "dev": dev,
           "stream": torch.cuda.Stream(dev), "pinned": pinned}

    head = run_workload(args.config, args, ctx, headline=True)
    records = {}
    for c in subs:
        try:
            records[c] = run_workload(c, args, ctx, headline=False)
        except Exception as exc:   # a record that fails is reported, the headline still prints
            if rank == 0:
                records[c] = {"error": f"{type(exc).__name__}: {str(exc)[:300]}"}
            if dist:
                raise

    if rank == 0:
        line = {"metric": METRIC, "value": head["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
                "scaling": head["scaling"], "vs_baseline": None, "dtype": DTYPE,
                "data": "synthetic (seeded GGUF superblocks)", "config": head["config"], "e2e": head["e2e"],
                "gpu_launches": head["gpu_launches"], "roofline": head["roofline"], "clocks": head["clocks"],
                "parity": head["parity"], "setup_s": head["setup_s"]}
        if "cpu_baseline" in head:
            line["cpu_baseline"] = head["cpu_baseline"]
        line["configs"] = records
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
