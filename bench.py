"""Benchmark of the MoE FFN layer (metric: MoE layer tok/s, with HBM GB/s and TFLOP/s against the
B200 roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl draco|reference]

One step = one MoE layer forward (routing, grouped expert gate/up/down, combine, shared expert
when the layer has one) over the configuration's token batch, synthetic seeded weights and
activations (dracomancer_llmengine_b200.synth).  Default workload: the second benchmark
configuration, chunked prefill of 512 tokens through the H2048/E128/top-8/F768 Q4_K+Q6_K layer on
one B200.

  value  device-resident throughput: inputs already in HBM, CUDA events on the launching
         stream (a dedicated non-default stream), weights (392 MB) larger than L2 so no flush
         is needed between steps.  Phase times (and the dominant kernel's, for the roofline)
         come from a second pass of the same steps with the library's per-phase events on.
  e2e    the same layer through the C ABI with pinned host X/out: the host->device copy of X and
         the device->host copy of the output are inside the timed region.

Under torchrun (N > 1) the layer runs expert-parallel (dracomancer_llmengine_b200.ep): each rank
holds E/N experts and its own batch of the configuration's token count (weak scaling: tokens per
GPU fixed), routes it, exchanges token rows with the expert owners by NCCL all-to-all, and adds
the returned partial rows and the shared expert at home; the time is the max over ranks and
`value` counts the tokens of all ranks.  `--impl reference` times the reference's own
CPU path of the layer on the host cores: routing restated from src/qwen35_prefill.py:180-188
(numpy) + the reference's m6_moe_tok with its fused AVX-512 GEMM (oracle/_ref, compiled from
the reference's sources); rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tok/s + HBM GB/s vs 8 TB/s (decode), TFLOP/s (prefill), 1-8 GPU"


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
                gateup_flops=2 * 2 * H * F * assign)


def profiled_traffic(config: str):
    """DRAM bytes per launch of the gate/up GEMM kernel from the committed ncu summary of this
    workload (profiles/tc_gemm_<config>.md, line `traffic_bytes_per_launch: N`), else None."""
    p = os.path.join(ROOT, "profiles", f"tc_gemm_{config}.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
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
        time.sleep(0.3)
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


def cpu_reference(layer, X, steps, warmup, budget_s=None):
    """The reference's CPU path on the host cores: numpy routing as in
    src/qwen35_prefill.py:180-188 (softmax) or the sigmoid/bias router of src/k2_numpy.py:57-71,
    then the reference's own m6_moe_tok (+ shared expert gemm when present)."""
    from oracle.oracle import Ref, Port, ref_available
    T = X.shape[0]
    K = layer.n_used
    if ref_available():
        R = Ref()
        kind = "reference"
    else:
        R = Port()
        kind = "port"
    gi = np.ascontiguousarray(layer.gate_inp)

    def route():
        lg = X @ gi.T
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

    def step():
        order, w = route()
        if kind == "reference":
            out = R.moe_tok(layer, X, order, w)
        else:
            out = R.moe_tok(layer, X, order, w)
        if layer.shared_inter:
            Port().shared_add(layer, X, out)
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2_prefill")
    ap.add_argument("--impl", default="draco", choices=["draco", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "fixed", "compact"],
                    help="expert-parallel token exchange (N > 1): peer-memory stores/loads with flag barriers, "
                         "or NCCL all-to-all with fixed blocks / exchanged counts")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    from dracomancer_llmengine_b200 import synth
    cfgd = synth.CONFIGS[args.config]
    T = cfgd["tokens"]
    config = {"workload": args.config, "hidden": cfgd["hidden"], "n_exp": cfgd["n_exp"], "top_k": cfgd["n_used"],
              "ffn": cfgd["inter"], "tokens_per_gpu": T, "formats": "Q4_K gate/up, Q6_K down",
              "shared_ffn": cfgd["shared_inter"], "routing": cfgd["scoring"],
              "l2": "weights and activations exceed L2 (no flush needed)" if args.config != "cfg1_decode"
              else "decode weights 25 MB fit in L2; flushed between steps by a 256 MB write then a 256 MB read"}

    if args.impl == "reference":
        if rank != 0:
            return
        layer, X = synth.make_config(args.config)
        steps = max(args.steps, 1)
        kind, times = cpu_reference(layer, X, steps, max(args.warmup, 1), budget_s=120)
        ms = statistics.median(times) * 1e3
        v = T / (ms / 1e3)
        cores = os.cpu_count()
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": 0, "steps": len(times),
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF superblocks)",
                "config": config, "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                                 "sample": f"{len(times)} full layer calls of {T} tokens (median)"},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    # page-locked staging buffers for the end-to-end leg, allocated first, as an engine would at
    # start-up (on the pool's VMs a later allocation of the same size copied ~1.5x slower)
    Xp = torch.empty((T, cfgd["hidden"]), dtype=torch.float32).pin_memory()
    Op = torch.empty((T, cfgd["hidden"]), dtype=torch.float32).pin_memory()
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import dracomancer_llmengine_b200 as dm
    L = dm.lib()

    # expert parallel: each rank generates (and uploads) only its own slice of the experts
    experts = (rank * (cfgd["n_exp"] // world), cfgd["n_exp"] // world) if world > 1 else None
    layer, Xh = synth.make_config(args.config, experts=experts)
    if rank:
        Xh = synth.make_tokens(layer, T, cfgd["seed"] + 1000 * rank, cfgd["zipf"])
    keep: list = []
    desc = dm.layer_desc(layer, keep) if world == 1 else None
    dev = torch.device("cuda", local)
    X = torch.from_numpy(Xh).to(dev)
    out = torch.empty((T, layer.hidden), device=dev, dtype=torch.float32)
    order = torch.empty((T, layer.n_used), device=dev, dtype=torch.int32)
    wtop = torch.empty((T, layer.n_used), device=dev, dtype=torch.float32)
    # a dedicated (non-default) stream, as an engine would give the library
    stream = torch.cuda.Stream(dev)
    import ctypes as ct
    ep = None
    if world > 1:
        from dracomancer_llmengine_b200.ep import ExpertParallelMoE
        with torch.cuda.stream(stream):
            ep = ExpertParallelMoE(layer, T, exchange=args.exchange, device=dev)

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

    # decode weights fit in L2: between steps write 256 MB (evicts them) and then read another
    # 256 MB, so the dirty lines of the write are written back before the step, not during it
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if args.config == "cfg1_decode" else None
    flush_r = torch.zeros(64 << 20, dtype=torch.float32, device=dev) if flush is not None else None

    def flush_l2():
        flush.zero_()
        flush_r.sum()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            fwd()
        if ep is not None and args.exchange == "p2p":
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
    experts = None
    if ep is not None:
        # every rank's routing, for the work of this rank's expert slice
        mine = ep._bufs["order"][:T].contiguous()
        allo = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allo, mine)
        order_h = torch.cat(allo).cpu().numpy()
        experts = (ep.ops.first, ep.ops.e_loc)
    else:
        order_h = order.cpu().numpy()
    work = layer_work(layer, order_h, T, experts)

    # ---- value: device-resident timed region ----
    launches0 = L.draco_b200_launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        for i in range(args.steps):
            if flush is not None:
                flush_l2()
            ev[i][0].record(stream)
            fwd()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    launches = L.draco_b200_launch_count() - launches0
    if graph is not None:   # replays bypass the host-side counter: the captured step's kernels
        launches = ep.launches_per_step * args.steps
    step_ms = [a.elapsed_time(b) for a, b in ev]
    # phase times (and the dominant kernel's) from a second pass of the same steps with the
    # library's per-phase CUDA events on, so the events do not inflate the timed steps
    dm.profile(True)
    g_saved, graph = graph, None   # per-phase events need the eager calls
    with torch.cuda.stream(stream):
        for i in range(args.steps):
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
    ms_per_step = tot_ms / args.steps
    value = world * T * args.steps / (tot_ms / 1e3)

    # ---- e2e: through the public API with pinned host buffers ----
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
    for _ in range(args.steps):
        fwd_host()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = world * T * args.steps / e2e_s

    # ---- roofline of the dominant kernel (gate/up grouped GEMM) ----
    hbm, bf16, src = peaks()
    gu_ms = prof["gateup"][0] / max(prof["gateup"][1], 1)
    gu_gbs = work["gateup_bytes"] / (gu_ms / 1e3) / 1e9
    roof = {"kernel": "gateup (grouped dequant GEMM, gate+up+SwiGLU)", "bound": "hbm", "achieved": gu_gbs,
            "peak": hbm, "unit": "GB/s", "frac": gu_gbs / hbm, "traffic": profiled_traffic(args.config) if world == 1 else None,
            "algorithmic_bytes": work["gateup_bytes"],
            "peak_source": src, "kernel_ms": gu_ms,
            "layer_gbs": work["bytes"] / (ms_per_step / 1e3) / 1e9,
            "layer_tflops": work["flops"] / (ms_per_step / 1e3) / 1e12,
            "phase_ms": {k: (v[0] / v[1] if v[1] else None) for k, v in prof.items()}}

    par = "single GPU"
    if world > 1:
        par = f"expert parallel x{world}: {layer.n_exp // world} experts/GPU, " + (
            "peer-memory exchange over NVLink" if args.exchange == "p2p" else f"NCCL all-to-all ({args.exchange})")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF superblocks)",
            "config": dict(config, parallelism=par, distinct_experts=work["distinct"]),
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": int(T * layer.hidden * 4),
                    "d2h_bytes_per_step": int(T * layer.hidden * 4)},
            "gpu_launches": int(launches), "roofline": roof, "clocks": clk.summary()}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        kind, times = cpu_reference(layer, Xh, steps=100, warmup=1, budget_s=20)
        cms = statistics.median(times) * 1e3
        line["cpu_baseline"] = {"value": T / (cms / 1e3), "unit": "tok/s", "cores": os.cpu_count(), "kind": kind,
                                "sample": f"{len(times)} full layer calls of {T} tokens, median, ~20 s budget"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ep is not None:
        ep.check()
        graph = None
        ep.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
