"""Expert parallelism for the MoE layer: one process per GPU, the E routed experts split
contiguously over the G ranks of a process group (rank r owns experts [r*E/G, (r+1)*E/G)), the
router and the shared expert replicated.

Two layouts:

* ``"a2a"`` (chunked prefill; every rank holds its own tokens).  Each rank routes its tokens with
  the full router, sends every token row once to each rank that owns one of its K experts, with
  the token's routing row beside it (all-to-all), the owners run their expert slice on the rows
  they received (the weighted sum over the token's experts that live there, k ascending), the
  partial rows travel back by the reverse all-to-all, and the home rank adds them in rank order
  and adds the shared expert it computed for its own tokens.  ``exchange="fixed"`` sends blocks
  of ``max_tokens`` rows to every rank (equal splits: no count exchange, no host round trip, the
  step can be captured in a CUDA graph); ``exchange="compact"`` exchanges the row counts first
  and sends only real rows (fewer bytes at large token counts, one host synchronisation);
  ``exchange="p2p"`` needs no collective at all: every rank maps the other ranks' receive and
  partial buffers (CUDA IPC), the pack kernel stores the token rows straight into the owners'
  receive buffers over NVLink, a flag barrier kernel (bounded wait) publishes them, the owners
  compute, a second barrier, and (``results="pull"``, the default) the home's combine kernel
  loads the result rows from the owners' memory; with ``results="push"`` the owners' combine
  kernel stores each result row straight into its home's partial buffer instead and the home
  adds its rows from its own memory (measured slower at 4 GPUs: 243 against 233 us per cfg2
  step, the peer stores lengthen the owners' combine by more than the home's loads take).
* ``"replicated"`` (decode; every rank holds the same tokens).  Each rank routes all tokens,
  runs its own experts on them (rank 0 adds the shared expert) and an all-reduce sums the
  partial outputs.

The reference engine is single-process; this is the expert-parallel form of its MoE layer
(src/m6_moe_tok.c:44-161 for the routed experts and the k-ordered combine, src/m6_layer.c:823-866
for the router).  The per-rank compute goes through an ``ops`` object: :class:`DeviceOps` runs
the CUDA library; tests substitute host implementations to check the exchange logic on CPU
process groups.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from . import DracoError, DracoMoeLayer, _check, _u64, _i, layer_desc, lib

LAYOUTS = ("a2a", "replicated")
EXCHANGES = ("fixed", "compact", "p2p")


def slice_desc(full: DracoMoeLayer, first: int, count: int, keep: list) -> DracoMoeLayer:
    """DracoMoeLayer for experts [first, first+count) of `full` (same shared expert, no router)."""
    ep = np.ctypeslib.as_array(full.exp_ptrs, shape=(3 * full.n_exp,))[3 * first:3 * (first + count)].copy()
    ec = np.ctypeslib.as_array(full.exp_codes, shape=(3 * full.n_exp,))[3 * first:3 * (first + count)].copy()
    keep += [ep, ec]
    d = DracoMoeLayer()
    for name, _ in DracoMoeLayer._fields_:
        setattr(d, name, getattr(full, name))
    d.n_exp = count
    d.exp_ptrs = ep.ctypes.data_as(_u64)
    d.exp_codes = ec.ctypes.data_as(_i)
    d.probs_b = None
    d.scoring, d.n_group, d.n_group_used = 0, 1, 1
    keep.append(d)
    return d


def tensor_at(ptr: int, shape, dtype, device):
    """A torch tensor over existing device memory (no copy; the memory must outlive it)."""
    import torch
    typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.int32: "<i4", torch.int64: "<i8",
               torch.uint32: "<u4"}[dtype]

    class _Cai:
        pass
    o = _Cai()
    o.__cuda_array_interface__ = {"shape": tuple(int(v) for v in shape), "typestr": typestr, "data": (ptr, False),
                                  "version": 3, "strides": None}
    return torch.as_tensor(o, device=device)


class PeerBuffers:
    """One rank's buffers of the peer-memory exchange, allocated by the library with CUDA IPC
    handles: receive rows x [G*B, H] (fp16 when x_half: the owners' tensor-core GEMMs round
    activations to fp16 in any case, so this halves the bytes on the links without changing a
    result), routing rows meta [G*B, 2K] int32, partial rows [G*B, H] fp32 and a control block
    (flag words [16] u32 at byte 0, barrier epoch at 64, status at 128).  `link` maps every
    rank's buffers and builds the device pointer arrays the kernels take."""
    CTL = 256

    def __init__(self, G, rank, B, H, K, device, x_half=True):
        import torch
        self.L, self.G, self.rank, self.device = lib(), G, rank, device
        self.B, self.H = B, H
        self.x_half = bool(x_half) and H % 8 == 0
        xb = 2 if self.x_half else 4
        sizes = {"x": G * B * H * xb, "meta": G * B * 2 * K * 4, "partial": G * B * H * 4, "ctl": self.CTL}
        self.own, self.handles, self.opened = {}, {}, []
        for name, n in sizes.items():
            p, h = ct.c_void_p(), (ct.c_char * 64)()
            _check(self.L.draco_b200_ep_mem_alloc(n, ct.byref(p), h), "draco_b200_ep_mem_alloc")
            self.own[name], self.handles[name] = p.value, bytes(h)
        self.x = tensor_at(self.own["x"], (G * B, H), torch.float16 if self.x_half else torch.float32, device)
        self.meta = tensor_at(self.own["meta"], (G * B, 2 * K), torch.int32, device)
        self.partial = tensor_at(self.own["partial"], (G * B, H), torch.float32, device)
        ctl = self.own["ctl"]
        self.my_flags, self.epoch, self.status = ctl, ctl + 64, ctl + 128
        self.status_t = tensor_at(self.status, (1,), torch.int32, device)

    def link(self, ptrs):
        """ptrs[r][name]: every rank's buffer addresses in this process."""
        import torch

        def arr(name, off=0):
            return torch.tensor([ptrs[r][name] + off for r in range(self.G)], dtype=torch.int64, device=self.device)
        self.dst_x, self.dst_meta = arr("x"), arr("meta")
        self.src_partial, self.peer_flags = arr("partial"), arr("ctl")
        # where this rank, as an owner, stores the results of the rows home h sent: row block
        # `rank` of h's partial buffer
        self.dst_partial = arr("partial", self.rank * self.B * self.H * 4)

    def open_peers(self, all_handles):
        """Map the other ranks' buffers from their handles (one process per GPU)."""
        ptrs = []
        for r, hs in enumerate(all_handles):
            if r == self.rank:
                ptrs.append(dict(self.own))
                continue
            d = {}
            for name, h in hs.items():
                q = ct.c_void_p()
                _check(self.L.draco_b200_ep_mem_open(h, ct.byref(q)), "draco_b200_ep_mem_open")
                d[name] = q.value
                self.opened.append(q.value)
            ptrs.append(d)
        self.link(ptrs)

    def close_peers(self):
        """Unmap the other ranks' buffers (waits for this device's work first)."""
        for p in self.opened:
            self.L.draco_b200_ep_mem_close(p)
        self.opened = []

    def free(self):
        """Release this rank's buffers; every rank must have unmapped them first."""
        for p in self.own.values():
            self.L.draco_b200_ep_mem_free(p)
        self.own = {}

    def close(self):
        self.close_peers()
        self.free()


class DeviceOps:
    """One rank's CUDA work (torch device tensors, asynchronous on the current torch stream)."""

    def __init__(self, layer, rank: int, world: int, device):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.keep: list = []
        self.full = layer_desc(layer, self.keep)
        self.e_loc = layer.n_exp // world
        self.first = rank * self.e_loc
        self.local = slice_desc(self.full, self.first, self.e_loc, self.keep)
        self.has_shared = bool(layer.shared_inter)
        self.L = lib()

    def _s(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def empty(self, shape, dtype):
        return self.torch.empty(shape, dtype=dtype, device=self.device)

    def route(self, x, T, order, wtop):
        _check(self.L.draco_b200_route(ct.byref(self.full), x.data_ptr(), T, order.data_ptr(), wtop.data_ptr(),
                                       self._s()), "draco_b200_route")

    def plan(self, order, T, K, E, G, block, counts, row_of, src_tok):
        _check(self.L.draco_b200_ep_plan(order.data_ptr(), T, K, E, G, block, counts.data_ptr(), row_of.data_ptr(),
                                         src_tok.data_ptr(), self._s()), "draco_b200_ep_plan")

    def pack(self, x, order, wtop, counts, G, src_tok, block, cap, K, H, send_x, send_meta):
        _check(self.L.draco_b200_ep_pack(x.data_ptr(), order.data_ptr(), wtop.data_ptr(), counts.data_ptr(), G,
                                         src_tok.data_ptr(), block, cap, K, H, send_x.data_ptr(),
                                         send_meta.data_ptr(), self._s()), "draco_b200_ep_pack")

    def shared(self, x, T, out):
        _check(self.L.draco_b200_experts_forward(ct.byref(self.local), x.data_ptr(), T, None, None, 0, 0,
                                                 out.data_ptr(), 1, 0, self._s()), "draco_b200_experts_forward")

    def _experts(self, x, T, order_ptr, wtop_ptr, ld, with_shared, out):
        x16 = 1 if x.dtype == self.torch.float16 else 0
        _check(self.L.draco_b200_experts_forward(ct.byref(self.local), x.data_ptr(), T, order_ptr, wtop_ptr, ld,
                                                 self.first, out.data_ptr(), 1 if with_shared else 0, x16,
                                                 self._s()), "draco_b200_experts_forward")

    def experts_routed(self, x, T, order, wtop, with_shared, out):
        """out[t] = sum_k wtop[t][k] * expert(x[t]) over the ids in this rank's slice (+ shared)."""
        self._experts(x, T, order.data_ptr(), wtop.data_ptr(), order.shape[1], with_shared, out)

    def experts_meta(self, x, R, meta, K, out):
        """The same on received rows (fp32, or fp16 from the peer-memory exchange) whose routing
        rows are {K ids, K weight bits} in meta [R, 2K]."""
        self._experts(x, R, meta.data_ptr(), meta.data_ptr() + 4 * K, 2 * K, False, out)

    def experts_to_homes(self, R, K, block, pb: "PeerBuffers"):
        """The received rows' results stored straight into the homes' partial buffers."""
        x16 = 1 if pb.x_half else 0
        _check(self.L.draco_b200_experts_forward_to_ranks(ct.byref(self.local), pb.x.data_ptr(), R, pb.meta.data_ptr(),
                                                          pb.meta.data_ptr() + 4 * K, 2 * K, self.first,
                                                          pb.dst_partial.data_ptr(), block, x16, self._s()),
               "draco_b200_experts_forward_to_ranks")

    def combine(self, back, row_of, T, G, H, sh, out):
        _check(self.L.draco_b200_ep_combine(back.data_ptr(), row_of.data_ptr(), T, G, H,
                                            sh.data_ptr() if sh is not None else None, out.data_ptr(), self._s()),
               "draco_b200_ep_combine")

    def push(self, x, order, wtop, counts, G, rank, src_tok, block, K, H, pb: PeerBuffers):
        _check(self.L.draco_b200_ep_push(x.data_ptr(), order.data_ptr(), wtop.data_ptr(), counts.data_ptr(), G, rank,
                                         src_tok.data_ptr(), block, K, H, pb.dst_x.data_ptr(), 1 if pb.x_half else 0,
                                         pb.dst_meta.data_ptr(), self._s()), "draco_b200_ep_push")

    def barrier(self, G, rank, pb: PeerBuffers):
        _check(self.L.draco_b200_ep_barrier(pb.peer_flags.data_ptr(), pb.my_flags, pb.epoch, G, rank, pb.status,
                                            self._s()), "draco_b200_ep_barrier")

    def pull_combine(self, row_of, T, G, rank, block, H, sh, out, pb: PeerBuffers):
        _check(self.L.draco_b200_ep_pull_combine(pb.src_partial.data_ptr(), row_of.data_ptr(), T, G, rank, block, H,
                                                 sh.data_ptr() if sh is not None else None, out.data_ptr(),
                                                 self._s()), "draco_b200_ep_pull_combine")


class TorchGroup:
    """The collectives of a torch.distributed process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_to_all(self, out, inp, out_splits=None, in_splits=None):
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def all_reduce(self, t):
        self.dist.all_reduce(t, group=self.group)

    def barrier(self):
        self.dist.barrier(group=self.group)

    def all_gather_object(self, obj):
        out = [None] * self.world
        self.dist.all_gather_object(out, obj, group=self.group)
        return out


class ExpertParallelMoE:
    """One rank of an expert-parallel MoE layer.  `layer` is the whole layer (synth.MoELayer-like:
    router, all experts' host weight buffers, shared expert); only this rank's slice of the
    experts is uploaded to its GPU.  `max_tokens` bounds the tokens of one call on any rank (all
    ranks must agree on it for the fixed exchange)."""

    def __init__(self, layer, max_tokens: int, comm=None, ops=None, layout: str = "a2a",
                 exchange: str = "fixed", device=None, results: str = "pull"):
        if layout not in LAYOUTS or exchange not in EXCHANGES or results not in ("push", "pull"):
            raise ValueError(f"layout in {LAYOUTS}, exchange in {EXCHANGES}, results in ('push', 'pull')")
        self.results = results
        self.comm = comm if comm is not None else TorchGroup()
        self.G, self.rank = self.comm.world, self.comm.rank
        if layer.n_exp % self.G:
            raise ValueError(f"{layer.n_exp} experts do not split over {self.G} ranks")
        if layer.n_exp // self.G < layer.n_used:
            raise ValueError("each rank needs at least n_used experts")
        self.layer = layer
        self.layout, self.exchange = layout, exchange
        self.ops = ops if ops is not None else DeviceOps(layer, self.rank, self.G, device)
        self.B = int(max_tokens)
        self.K, self.H, self.E = layer.n_used, layer.hidden, layer.n_exp
        self._bufs = None

    # ---- buffers (allocated once: stable addresses let the library replay its launch graphs) ----
    def _alloc(self):
        import torch
        o, B, G, K, H = self.ops, self.B, self.G, self.K, self.H
        f32, i32 = torch.float32, torch.int32
        b = {"order": o.empty((B, K), i32), "wtop": o.empty((B, K), f32), "out": o.empty((B, H), f32)}
        if self.layout == "a2a":
            cap = G * B if self.exchange != "compact" else B * min(K, G)
            rcap = G * B
            b.update(counts=o.empty((G,), i32), rcounts=o.empty((G,), i32), row_of=o.empty((B, G), i32),
                     src_tok=o.empty((max(cap, 1),), i32), send_x=o.empty((cap, H), f32),
                     send_meta=o.empty((cap, 2 * K), i32), recv_x=o.empty((rcap, H), f32),
                     recv_meta=o.empty((rcap, 2 * K), i32), partial=o.empty((rcap, H), f32),
                     back=o.empty((cap, H), f32), sh=o.empty((B, H), f32) if o.has_shared else None)
            b["cap"] = cap
            if self.exchange == "p2p":
                for k in ("send_x", "send_meta", "recv_x", "recv_meta", "partial", "back", "rcounts"):
                    b[k] = None
                self.peer = PeerBuffers(G, self.rank, B, H, K, o.device)
                if G == 1:
                    self.peer.link([dict(self.peer.own)])
                elif hasattr(self.comm, "all_gather_object"):
                    self.peer.open_peers(self.comm.all_gather_object(self.peer.handles))
        self._bufs = b
        return b

    def capture(self, x, out):
        """A CUDA graph of forward(x, out) for fixed buffers x and out (the peer-memory exchange:
        no collective library call and no host round trip in the step), after one eager call
        that sizes every workspace.  Returns the torch.cuda.CUDAGraph; replay() runs the step on
        the current contents of x.  Graphs cannot hold the host synchronisation of the "compact"
        exchange or the NCCL collectives of "fixed" and "replicated" here."""
        import torch
        if self.exchange != "p2p" or self.layout != "a2a":
            raise ValueError("capture needs the peer-memory exchange")
        n0 = lib().draco_b200_launch_count()
        self.forward(x, out)
        # the library's kernels in one step (a replay launches the same ones without the host)
        self.launches_per_step = int(lib().draco_b200_launch_count() - n0)
        torch.cuda.current_stream().synchronize()
        g = torch.cuda.CUDAGraph()
        # thread-local capture: other threads of the process (a process group's watchdog) keep
        # using CUDA while this one captures
        with torch.cuda.graph(g, stream=torch.cuda.current_stream(), capture_error_mode="thread_local"):
            self.forward(x, out)
        return g

    def check(self):
        """Raise if a barrier of the peer-memory exchange gave up waiting (status read back)."""
        if self.exchange == "p2p" and self._bufs is not None:
            st = int(self.peer.status_t.item())
            if st:
                raise DracoError(f"expert-parallel barrier timed out on rank {self.rank} (status 0x{st:x})")

    def close(self):
        """Release the peer-memory buffers (collective over the group when it has a barrier)."""
        if getattr(self, "peer", None) is not None:
            self.peer.close_peers()
            if hasattr(self.comm, "barrier"):
                self.comm.barrier()
            self.peer.free()
            self.peer = None

    def forward(self, x, out=None):
        """MoE layer output for this rank's token rows x [T, H] (fp32).  With layout "replicated"
        every rank passes the same x and gets the same output."""
        T = int(x.shape[0])
        if T > self.B:
            raise ValueError(f"{T} tokens > max_tokens {self.B}")
        b = self._bufs or self._alloc()
        if out is None:
            out = b["out"][:T]
        if T == 0:
            x = b["out"]   # a rank without tokens still takes part in the exchange; nothing reads x
        if self.layout == "replicated":
            return self._forward_replicated(x, T, b, out)
        if self.exchange == "p2p":
            return self._forward_p2p(x, T, b, out)
        return self._forward_a2a(x, T, b, out)

    def _forward_p2p(self, x, T, b, out):
        o, G, K, H, E, B, pb = self.ops, self.G, self.K, self.H, self.E, self.B, self.peer
        o.route(x, T, b["order"], b["wtop"])
        o.plan(b["order"], T, K, E, G, B, b["counts"], b["row_of"], b["src_tok"])
        sh = None
        if o.has_shared:
            sh = b["sh"][:T]
            o.shared(x, T, sh)
        o.push(x, b["order"], b["wtop"], b["counts"], G, self.rank, b["src_tok"], B, K, H, pb)
        o.barrier(G, self.rank, pb)                 # every rank's rows have landed
        if self.results == "push":
            o.experts_to_homes(G * B, K, B, pb)     # results stored into the homes' partial rows
            o.barrier(G, self.rank, pb)             # every owner's results have landed
            o.combine(pb.partial, b["row_of"], T, G, H, sh, out)
            return out
        o.experts_meta(pb.x, G * B, pb.meta, K, pb.partial)
        o.barrier(G, self.rank, pb)                 # every owner's partial rows are final
        o.pull_combine(b["row_of"], T, G, self.rank, B, H, sh, out, pb)
        return out

    def _forward_replicated(self, x, T, b, out):
        o = self.ops
        order, wtop = b["order"][:T], b["wtop"][:T]
        o.route(x, T, order, wtop)
        o.experts_routed(x, T, order, wtop, o.has_shared and self.rank == 0, out)
        self.comm.all_reduce(out)
        return out

    def _forward_a2a(self, x, T, b, out):
        o, G, K, H, E, B = self.ops, self.G, self.K, self.H, self.E, self.B
        fixed = self.exchange == "fixed"
        block = B if fixed else 0
        cap = b["cap"]
        o.route(x, T, b["order"], b["wtop"])
        o.plan(b["order"], T, K, E, G, block, b["counts"], b["row_of"], b["src_tok"])
        o.pack(x, b["order"], b["wtop"], b["counts"], G, b["src_tok"], block, cap, K, H, b["send_x"],
               b["send_meta"])
        sh = None
        if o.has_shared:
            sh = b["sh"][:T]
            o.shared(x, T, sh)
        if fixed:
            S = R = G * B
            send_x, send_meta, sc, rc = b["send_x"], b["send_meta"], None, None
            recv_x, recv_meta = b["recv_x"], b["recv_meta"]
        else:
            self.comm.all_to_all(b["rcounts"], b["counts"])
            sc, rc = [int(v) for v in b["counts"].tolist()], [int(v) for v in b["rcounts"].tolist()]
            S, R = sum(sc), sum(rc)
            send_x, send_meta = b["send_x"][:S], b["send_meta"][:S]
            recv_x, recv_meta = b["recv_x"][:R], b["recv_meta"][:R]
        self.comm.all_to_all(recv_x, send_x, rc, sc)
        self.comm.all_to_all(recv_meta, send_meta, rc, sc)
        partial = b["partial"][:R]
        if R:
            o.experts_meta(recv_x, R, recv_meta, K, partial)
        back = b["back"][:S]
        self.comm.all_to_all(back, partial, sc, rc)
        o.combine(back, b["row_of"], T, G, H, sh, out)
        return out


def emulate_p2p(ranks: list, xs: list) -> list:
    """The peer-memory exchange of G ranks that share one GPU in one process: the ranks' buffers
    are linked directly, and the steps run rank after rank in one stream, which orders them the
    way the barriers do across GPUs (no barrier kernel runs: ranks on one GPU must not wait on
    one another in separate launches)."""
    G = len(ranks)
    assert all(r.G == G and r.exchange == "p2p" for r in ranks)
    for r in ranks:
        if r._bufs is None:
            r._alloc()
    ptrs = [dict(r.peer.own) for r in ranks]
    for r in ranks:
        r.peer.link(ptrs)
    sts = []
    for r, x in zip(ranks, xs):
        o, b, T = r.ops, r._bufs, int(x.shape[0])
        if T == 0:
            x = b["out"]
        o.route(x, T, b["order"], b["wtop"])
        o.plan(b["order"], T, r.K, r.E, G, r.B, b["counts"], b["row_of"], b["src_tok"])
        sh = None
        if o.has_shared:
            sh = b["sh"][:T]
            o.shared(x, T, sh)
        o.push(x, b["order"], b["wtop"], b["counts"], G, r.rank, b["src_tok"], r.B, r.K, r.H, r.peer)
        sts.append((T, sh))
    for r in ranks:
        if r.results == "push":
            r.ops.experts_to_homes(G * r.B, r.K, r.B, r.peer)
        else:
            r.ops.experts_meta(r.peer.x, G * r.B, r.peer.meta, r.K, r.peer.partial)
    outs = []
    for r, (T, sh) in zip(ranks, sts):
        out = r._bufs["out"][:T]
        if r.results == "push":
            r.ops.combine(r.peer.partial, r._bufs["row_of"], T, G, r.H, sh, out)
        else:
            r.ops.pull_combine(r._bufs["row_of"], T, G, r.rank, r.B, r.H, sh, out, r.peer)
        outs.append(out)
    return outs


def emulate(ranks: list, xs: list) -> list:
    """Run the a2a layout of several ExpertParallelMoE ranks that live in one process (one GPU or
    CPU) with the exchanges done by copies: the data path of G ranks without G devices.  The
    ranks' `comm` objects are not used."""
    import torch
    G = len(ranks)
    assert all(r.G == G and r.layout == "a2a" for r in ranks)
    if ranks[0].exchange == "p2p":
        return emulate_p2p(ranks, xs)
    st = []
    for r, x in zip(ranks, xs):
        o, b = r.ops, r._bufs or r._alloc()
        T = int(x.shape[0])
        if T == 0:
            x = b["out"]
        block = r.B if r.exchange == "fixed" else 0
        o.route(x, T, b["order"], b["wtop"])
        o.plan(b["order"], T, r.K, r.E, G, block, b["counts"], b["row_of"], b["src_tok"])
        o.pack(x, b["order"], b["wtop"], b["counts"], G, b["src_tok"], block, b["cap"], r.K, r.H, b["send_x"],
               b["send_meta"])
        sh = None
        if o.has_shared:
            sh = b["sh"][:T]
            o.shared(x, T, sh)
        st.append((T, [int(v) for v in b["counts"].tolist()], sh))

    def seg(i, d):   # rows rank i sends to rank d
        r, (T, cnt, _) = ranks[i], st[i]
        if r.exchange == "fixed":
            return r.B * d, r.B
        return sum(cnt[:d]), cnt[d]

    partials = []
    for d, r in enumerate(ranks):
        rx = torch.cat([ranks[i]._bufs["send_x"][seg(i, d)[0]:sum(seg(i, d))] for i in range(G)])
        rm = torch.cat([ranks[i]._bufs["send_meta"][seg(i, d)[0]:sum(seg(i, d))] for i in range(G)])
        R = int(rx.shape[0])
        part = r.ops.empty((R, r.H), torch.float32)
        if R:
            r.ops.experts_meta(rx, R, rm, r.K, part)
        partials.append(part)
    outs = []
    for i, r in enumerate(ranks):
        T, cnt, sh = st[i]
        back_parts = []
        for d in range(G):
            # rows of rank i inside rank d's received buffer start after ranks < i
            off = sum(seg(j, d)[1] for j in range(i))
            back_parts.append(partials[d][off:off + seg(i, d)[1]])
        back = torch.cat(back_parts)
        out = r.ops.empty((T, r.H), torch.float32)
        r.ops.combine(back, r._bufs["row_of"], T, G, r.H, sh, out)
        outs.append(out)
    return outs


__all__ = ["ExpertParallelMoE", "DeviceOps", "PeerBuffers", "TorchGroup", "emulate", "emulate_p2p", "slice_desc",
           "tensor_at", "DracoError"]
