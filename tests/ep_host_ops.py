"""Host (CPU) restatement of one expert-parallel rank's work, with the interface of
dracomancer_llmengine_b200.ep.DeviceOps, for checking the exchange logic on CPU process groups
and the CUDA exchange kernels against it.  Test infrastructure: the compute goes through the
oracle (oracle/moe_oracle.c), the plan/pack/combine are plain loops."""
import numpy as np
import torch


def plan_ref(order, E, G, block):
    """(counts[G], row_of[T, G], src_tok[rows]) of the expert-parallel send plan: a token sends one
    row to each rank that owns one of its experts; rank-major rows, tokens ascending within a
    rank; rank r's rows start at r*block (block > 0) or after rank r-1's (block == 0)."""
    order = np.asarray(order)
    T = order.shape[0]
    e_loc = E // G
    counts = np.zeros(G, np.int32)
    row_of = np.full((T, G), -1, np.int32)
    cap = G * block if block else T * min(order.shape[1], G)
    src_tok = np.full(max(cap, 1), -1, np.int32)
    base = 0
    for r in range(G):
        start = r * block if block else base
        n = 0
        for t in range(T):
            if any(0 <= e < E and e // e_loc == r for e in order[t]):
                row_of[t, r] = start + n
                src_tok[start + n] = t
                n += 1
        counts[r] = n
        base = start + n
    return counts, row_of, src_tok


class HostOps:
    def __init__(self, layer, rank, world, port):
        self.layer, self.port = layer, port
        self.e_loc = layer.n_exp // world
        self.first = rank * self.e_loc
        self.has_shared = bool(layer.shared_inter)

    def empty(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype)

    def route(self, x, T, order, wtop):
        o, w = self.port.route(self.layer, x[:T].numpy())
        order[:T] = torch.from_numpy(o)
        wtop[:T] = torch.from_numpy(w)

    def plan(self, order, T, K, E, G, block, counts, row_of, src_tok):
        c, ro, st = plan_ref(order[:T].numpy(), E, G, block)
        counts[:] = torch.from_numpy(c)
        row_of[:T] = torch.from_numpy(ro)
        src_tok[:st.size] = torch.from_numpy(st)

    def pack(self, x, order, wtop, counts, G, src_tok, block, cap, K, H, send_x, send_meta):
        c = counts.numpy()
        rows = [(r * block + j) if block else (int(c[:r].sum()) + j) for r in range(G) for j in range(int(c[r]))]
        if block:
            for row in range(min(G * block, cap)):
                send_meta[row, :K] = -1
                send_meta[row, K:] = 0
        for row in rows:
            if row >= cap:
                continue
            t = int(src_tok[row])
            send_x[row] = x[t]
            send_meta[row, :K] = order[t]
            send_meta[row, K:] = wtop[t].view(torch.int32)

    def shared(self, x, T, out):
        acc = np.zeros((T, self.layer.hidden), np.float32)
        self.port.shared_add(self.layer, x[:T].numpy(), acc)
        out[:T] = torch.from_numpy(acc)

    def experts_routed(self, x, T, order, wtop, with_shared, out):
        o = np.array(order[:T].numpy(), np.int32)
        o[(o < self.first) | (o >= self.first + self.e_loc)] = -1
        y = self.port.moe_tok(self.layer, x[:T].numpy(), o, wtop[:T].numpy())
        if with_shared:
            self.port.shared_add(self.layer, x[:T].numpy(), y)
        out[:T] = torch.from_numpy(y)

    def experts_meta(self, x, R, meta, K, out):
        self.experts_routed(x, R, meta[:R, :K].contiguous(), meta[:R, K:].contiguous().view(torch.float32),
                            False, out)

    def combine(self, back, row_of, T, G, H, sh, out):
        acc = np.zeros((T, H), np.float32)
        b = back.numpy()
        ro = row_of[:T].numpy()
        for r in range(G):
            for t in range(T):
                if ro[t, r] >= 0:
                    acc[t] += b[ro[t, r]]
        if sh is not None:
            acc += sh[:T].numpy()
        out[:T] = torch.from_numpy(acc)
