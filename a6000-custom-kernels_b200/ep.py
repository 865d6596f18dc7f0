"""Expert parallelism for MoE decode and prefill.

Each rank holds a contiguous 1/world of every layer's experts (the reference's
cache is single-GPU; the partition follows the expert-major tensor layout, so a
rank's experts are one contiguous slice of each tensor).

Decode: every rank routes the same tokens over ALL experts (replicated logits
and activations: at decode batch sizes that is a few KB), runs the GEMVs on
the picks it holds (moe_b200_ep_layer_decode), and the ranks sum their shares
of the weighted combine with one all-reduce (NCCL over NVLink on GPUs, gloo on
CPU). The shared expert runs on rank 0 only.

Prefill: every rank routes its OWN tokens, sorts its (token, pick) entries by
the rank owning the picked expert, and an all-to-all sends each entry's
activation row and local expert id there (dispatch); each rank runs the
tensor-core expert prefill on the rows it received (moe_b200_experts_prefill,
one pick per row), a second all-to-all returns the outputs (combine), and the
source rank adds its shared expert and the weighted sum. The data movement
(sort, row gather / scatter, all-to-all) is torch plumbing; every product runs
in libmoe_b200.so.
"""
import ctypes

import torch

from ._lib import MoeLayerDesc, check, lib
from .moe_cache import _ptr, _stream, expert_tensor, topk_softmax


def expert_range(n_experts, rank, world):
    """Global experts [lo, hi) held by `rank` of `world` (contiguous, balanced)."""
    return n_experts * rank // world, n_experts * (rank + 1) // world


class EPMoELayer:
    """This rank's share of one MoE layer. Built from a full MoELayer (same
    weights as the single-GPU layer) by slicing its expert tensors (the full
    tensors are not kept), or with local=True from a MoELayer that already
    holds only this rank's experts [lo, hi) of n_experts."""

    def __init__(self, full, rank, world, group=None, local=False, n_experts=None):
        self.H, self.F, self.k = full.H, full.F, full.k
        self.E = n_experts if local else full.E
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = expert_range(self.E, rank, world)
        self.device = full.device
        self.types = dict(full.types)
        self.norm_w = full.norm_w
        shapes = {"gate": (full.F, full.H), "up": (full.F, full.H), "down": (full.H, full.F)}
        if local:
            assert full.E == self.hi - self.lo
            self.w = dict(full.w)
        else:
            self.w = {r: full.w[r][self.lo:self.hi].clone() for r in ("gate", "up", "down")}
        self.shared = dict(full.shared)
        self.desc_t = {r: expert_tensor(self.w[r], self.types[r], shapes[r][1], shapes[r][0],
                                        name=f"{full.desc_t[r].name.decode()}.ep{rank}")
                       for r in ("gate", "up", "down")}
        d = MoeLayerDesc()
        d.gate, d.up, d.down = self.desc_t["gate"], self.desc_t["up"], self.desc_t["down"]
        d.shared_type = full.desc.shared_type
        d.shared_gate = _ptr(self.shared.get("gate"))
        d.shared_up = _ptr(self.shared.get("up"))
        d.shared_down = _ptr(self.shared.get("down"))
        d.H, d.F, d.n_experts, d.k = full.H, full.F, self.hi - self.lo, full.k
        d.glu_op, d.glu_limit, d.norm_w = full.desc.glu_op, full.desc.glu_limit, full.desc.norm_w
        self.desc = d
        self._ws = {}

    def workspace(self, n_tok):
        ws = self._ws.get(n_tok)
        if ws is None:
            nbytes = lib().moe_b200_layer_workspace_size(ctypes.byref(self.desc), n_tok)
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[n_tok] = ws
        return ws

    def partial(self, x, logits, out=None, stream=None):
        """This rank's share of the layer output (no communication)."""
        n_tok = x.shape[0]
        if out is None:
            out = torch.empty((n_tok, self.H), dtype=torch.float32, device=self.device)
        ws = self.workspace(n_tok)
        check(lib().moe_b200_ep_layer_decode(ctypes.byref(self.desc), self.lo, self.E, 1 if self.rank == 0 else 0,
                                             _ptr(x), _ptr(logits), _ptr(out), n_tok, _ptr(ws), ws.numel(),
                                             _stream(stream)))
        return out

    def decode(self, x, logits, out=None, stream=None):
        """The full layer output on every rank: shares summed by all-reduce."""
        import torch.distributed as dist
        out = self.partial(x, logits, out, stream)
        if self.world > 1:
            with torch.cuda.stream(stream) if stream is not None else _null():
                dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out

    def decode_p2p(self, ex, x, logits, out=None, stream=None):
        """This rank's token through the layer with the experts sharded over
        the ranks and the exchange inside the layer kernel
        (moe_b200_ep_layer_decode_p2p): x f32 [1, H], logits f32 [1, E]
        (device) -> out f32 [1, H]. `ex` is a connected DecodeExchange."""
        if out is None:
            out = torch.empty((1, self.H), dtype=torch.float32, device=self.device)
        ws = self.workspace(self.world)
        check(lib().moe_b200_ep_layer_decode_p2p(ctypes.byref(self.desc), self.lo, self.E, ex.table, self.world,
                                                 self.rank, _ptr(x), _ptr(logits), _ptr(out), _ptr(ws), ws.numel(),
                                                 _stream(stream)))
        return out

    # ---- prefill ------------------------------------------------------------
    def _prefill_ws(self, n_tok, k):
        key = ("prefill", n_tok, k)
        ws = self._ws.get(key)
        if ws is None:
            nbytes = lib().moe_b200_experts_prefill_workspace_size(ctypes.byref(self.desc), max(1, n_tok), k)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def route(self, logits, stream=None):
        """Top-k over all experts of this rank's tokens: (ids, weights) [n, k]."""
        return topk_softmax(logits, self.k, self.norm_w, stream=stream)

    def dispatch_plan(self, ids):
        return dispatch_plan(ids, self.E, self.world)

    def experts(self, x_rows, local_ids, stream=None):
        """y [n, H] for rows that picked local expert local_ids[i] (one pick per row)."""
        n = x_rows.shape[0]
        y = torch.empty((n, self.H), dtype=torch.float32, device=self.device)
        if n == 0:
            return y
        ws = self._prefill_ws(n, 1)
        check(lib().moe_b200_experts_prefill(ctypes.byref(self.desc), _ptr(x_rows), 0, _ptr(local_ids), n, 1,
                                             _ptr(y), _ptr(ws), ws.numel(), _stream(stream)))
        return y

    def finish(self, x, w, y, out=None, stream=None):
        """out = sum_p w[t][p] y[t][p] (+ the shared expert of x)."""
        n = x.shape[0]
        if out is None:
            out = torch.empty((n, self.H), dtype=torch.float32, device=self.device)
        ys = None
        if self.shared:
            ys = torch.empty((n, self.H), dtype=torch.float32, device=self.device)
            ws = self._prefill_ws(n, self.k)
            check(lib().moe_b200_shared_prefill(ctypes.byref(self.desc), _ptr(x), n, _ptr(ys), _ptr(ws), ws.numel(),
                                                _stream(stream)))
        check(lib().moe_b200_combine(_ptr(y), _ptr(w), _ptr(ys), _ptr(out), n, self.H, self.k, _stream(stream)))
        return out

    def prefill(self, x, logits, out=None, stream=None):
        """This rank's tokens through the layer with the experts spread over the
        ranks: route, dispatch all-to-all, local expert prefill, combine
        all-to-all, shared expert and weighted sum."""
        ids, w = self.route(logits, stream)
        y = exchange(x, ids, self.E, self.world, lambda rows, lids: self.experts(rows, lids, stream), self.group)
        return self.finish(x, w, y, out, stream)


def dispatch_plan(ids, n_experts, world):
    """A rank's entries (t, p) in owner-rank order: (order, send_counts, local
    expert ids in that order); order[i] = t * k + p of the i-th entry sent."""
    bounds = torch.tensor([expert_range(n_experts, r, world)[1] for r in range(world)], device=ids.device,
                          dtype=torch.int64)
    flat = ids.reshape(-1).to(torch.int64)
    owner = torch.bucketize(flat, bounds, right=True)
    order = torch.argsort(owner, stable=True)
    counts = torch.bincount(owner, minlength=world)
    lo = torch.tensor([expert_range(n_experts, r, world)[0] for r in range(world)], device=ids.device,
                      dtype=torch.int64)
    local = (flat - lo[owner])[order].to(torch.int32)
    return order, counts, local


def exchange(x, ids, n_experts, world, compute, group=None):
    """Dispatch / combine of one layer's expert work: sends each entry's row
    x[t] and local expert id to the owning rank (all-to-all), runs
    compute(rows, local_ids) -> [rows, H] there, returns the outputs (second
    all-to-all) and puts them back in entry order: y [n, k, H]."""
    import torch.distributed as dist
    n, k = ids.shape
    order, send_counts, local = dispatch_plan(ids, n_experts, world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    x_send = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
    x_recv = torch.empty((sum(rc), x.shape[1]), dtype=x.dtype, device=x.device)
    ids_recv = torch.empty((sum(rc),), dtype=torch.int32, device=x.device)
    dist.all_to_all_single(x_recv, x_send, rc, sc, group=group)
    dist.all_to_all_single(ids_recv, local, rc, sc, group=group)
    y_recv = compute(x_recv, ids_recv)
    H = y_recv.shape[1]
    y_back = torch.empty((n * k, H), dtype=y_recv.dtype, device=x.device)
    dist.all_to_all_single(y_back, y_recv, sc, rc, group=group)
    y = torch.empty_like(y_back)
    y[order] = y_back
    return y.view(n, k, H)


class PeerExchange:
    """One GPU's buffers for the expert-parallel prefill exchange over NVLink
    peer memory, and the other GPUs' (opened by CUDA IPC): received rows x
    [W * cap][H], their local expert ids and source entries [W * cap], the
    outputs of this GPU's own entries y_ret [cap][H], arrival counters [2].
    cap = the entries one GPU sends per layer (prompt tokens x k). With
    `local_peers` (ranks emulated in one process on one GPU) the other ranks'
    buffers are used directly instead of IPC."""

    NAMES = ("x", "ids", "src", "y_ret", "flags")

    def __init__(self, H, cap, rank, world, group=None, local_peers=None):
        self.H, self.cap, self.rank, self.world = H, cap, rank, world
        sizes = {"x": 4 * world * cap * H, "ids": 4 * world * cap, "src": 4 * world * cap, "y_ret": 4 * cap * H,
                 "flags": 256}
        self.own = {}
        for name in self.NAMES:
            p = ctypes.c_void_p()
            check(lib().moe_b200_ipc_alloc(sizes[name], ctypes.byref(p)))
            self.own[name] = p.value
        p = ctypes.c_void_p()
        check(lib().moe_b200_ipc_alloc(64, ctypes.byref(p)))
        self.scratch = p.value
        self.opened = []
        self.local_peers = local_peers
        self.calls = 0
        self.group = group

    def connect(self, peers=None):
        """Build the [5][W] pointer table: IPC handles over the process group,
        or the emulated ranks' own buffers."""
        W = self.world
        table = [[0] * W for _ in self.NAMES]
        if peers is not None:
            for r, ex in enumerate(peers):
                for i, name in enumerate(self.NAMES):
                    table[i][r] = ex.own[name]
        else:
            import torch.distributed as dist
            mine = {}
            for name in self.NAMES:
                h = (ctypes.c_char * 64)()
                check(lib().moe_b200_ipc_handle(self.own[name], h))
                mine[name] = bytes(h)
            every = [None] * W
            dist.all_gather_object(every, mine, group=self.group)
            for r in range(W):
                for i, name in enumerate(self.NAMES):
                    if r == self.rank:
                        table[i][r] = self.own[name]
                    else:
                        p = ctypes.c_void_p()
                        h = (ctypes.c_char * 64).from_buffer_copy(every[r][name])
                        check(lib().moe_b200_ipc_open(h, ctypes.byref(p)))
                        self.opened.append(p.value)
                        table[i][r] = p.value
        self.table = (ctypes.c_void_p * (5 * W))(*[v for row in table for v in row])
        return self

    def close(self):
        for p in self.opened:
            lib().moe_b200_ipc_close(p)
        self.opened = []
        for p in list(self.own.values()) + [self.scratch]:
            lib().moe_b200_ipc_free(p)
        self.own = {}


class DecodeExchange:
    """One GPU's buffer of the expert-parallel decode exchange (gather slots
    for every GPU's token, the returned down rows of this GPU's token, arrival
    and row counters; layout in include/moe_cache_b200.h), and the other
    GPUs' buffers opened by CUDA IPC. One exchange serves any number of layers
    of one shape, called in the same order on every GPU."""

    def __init__(self, H, n_experts, k, rank, world, group=None):
        self.rank, self.world, self.group = rank, world, group
        nbytes = lib().moe_b200_ep_decode_buffer_bytes(H, n_experts, k, world)
        if nbytes == 0:
            raise ValueError("bad expert-parallel decode shape")
        p = ctypes.c_void_p()
        check(lib().moe_b200_ipc_alloc(nbytes, ctypes.byref(p)))
        self.own = p.value
        self.opened = []
        self.table = None

    def connect(self):
        W = self.world
        ptrs = [0] * W
        ptrs[self.rank] = self.own
        if W > 1:
            import torch.distributed as dist
            h = (ctypes.c_char * 64)()
            check(lib().moe_b200_ipc_handle(self.own, h))
            every = [None] * W
            dist.all_gather_object(every, bytes(h), group=self.group)
            for r in range(W):
                if r == self.rank:
                    continue
                p = ctypes.c_void_p()
                check(lib().moe_b200_ipc_open((ctypes.c_char * 64).from_buffer_copy(every[r]), ctypes.byref(p)))
                self.opened.append(p.value)
                ptrs[r] = p.value
        self.table = (ctypes.c_void_p * W)(*ptrs)
        return self

    def close(self):
        for p in self.opened:
            check(lib().moe_b200_ipc_close(p))
        self.opened = []
        if self.own:
            check(lib().moe_b200_ipc_free(self.own))
            self.own = None


def prefill_p2p_stages(L, ex, x, logits, stream=None):
    """Stage 1 of a layer on one rank: route and dispatch (peer stores)."""
    n, k = x.shape[0], L.k
    assert n * k <= ex.cap
    ids, w = L.route(logits, stream)
    check(lib().moe_b200_ep_dispatch(ex.table, L.world, L.rank, ex.cap, _ptr(ids), n * k, k, L.E, _ptr(x), L.H,
                                     ex.scratch, _stream(stream)))
    ex.calls += 1
    return w


def _ep_rows(L, ex, stream=None):
    """Stage 2 on an owner: its experts on every received row, outputs back."""
    W, rows = L.world, L.world * ex.cap
    key = ("rows", rows)
    bufs = L._ws.get(key)
    if bufs is None:
        nbytes = lib().moe_b200_ep_experts_rows_workspace_size(ctypes.byref(L.desc), rows)
        bufs = (torch.empty(nbytes, dtype=torch.uint8, device=L.device),
                torch.empty((rows, L.F), dtype=torch.float32, device=L.device),
                torch.empty((rows, L.F), dtype=torch.float32, device=L.device),
                torch.empty((rows, L.H), dtype=torch.float32, device=L.device))
        L._ws[key] = bufs
    ws, g, u, y = bufs
    check(lib().moe_b200_ep_experts_rows(ctypes.byref(L.desc), ex.own["x"], ex.own["ids"], rows, _ptr(g), _ptr(u),
                                         _ptr(y), _ptr(ws), ws.numel(), _stream(stream)))
    check(lib().moe_b200_ep_return(ex.table, W, ex.cap, ex.own["ids"], ex.own["src"], _ptr(y), L.H, ex.scratch,
                                   _stream(stream)))


def prefill_p2p(L, ex, x, logits, out=None, stream=None):
    """One layer of the expert-parallel prefill with the exchange over peer
    memory: route, dispatch, wait for every GPU's rows, the owned experts on
    them, return, wait for every owner's outputs, shared expert and combine.
    Nothing waits on the host: the stream carries every dependency."""
    w = prefill_p2p_stages(L, ex, x, logits, stream)
    target = L.world * ex.calls
    check(lib().moe_b200_ep_wait(ex.own["flags"], target, _stream(stream)))
    _ep_rows(L, ex, stream)
    check(lib().moe_b200_ep_wait(ex.own["flags"] + 4, target, _stream(stream)))
    n = x.shape[0]
    return L.finish(x, w, ex.own["y_ret"], out, stream)


def prefill_p2p_emulated(ranks, exs, xs, logits):
    """prefill_p2p of len(ranks) ranks in ONE process on one GPU, stage by
    stage over all ranks (every dispatch before any owner reads, every return
    before any source combines), so no wait is left pending."""
    ws_ = [prefill_p2p_stages(L, ex, xs[r], logits[r]) for r, (L, ex) in enumerate(zip(ranks, exs))]
    for L, ex in zip(ranks, exs):
        _ep_rows(L, ex)
    return [L.finish(xs[r], ws_[r], ex.own["y_ret"]) for r, (L, ex) in enumerate(zip(ranks, exs))]


def prefill_emulated(ranks, xs, logits):
    """The expert-parallel prefill of len(ranks) ranks in ONE process (one GPU):
    the all-to-alls become slicing; every other step is the ranks' own. For
    tests of the dispatch / combine logic without several GPUs."""
    W = len(ranks)
    plans, ws_ = [], []
    for r, L in enumerate(ranks):
        ids, w = L.route(logits[r])
        order, counts, local = L.dispatch_plan(ids)
        plans.append((order, counts.tolist(), local))
        ws_.append(w)
    # dispatch: rank d receives, from each source s in rank order, s's slice for d
    offs = [[sum(plans[s][1][:d]) for d in range(W)] for s in range(W)]
    y_parts = [[None] * W for _ in range(W)]
    for d, L in enumerate(ranks):
        rows, lids, src = [], [], []
        for s in range(W):
            order, counts, local = plans[s]
            a, b = offs[s][d], offs[s][d] + counts[d]
            rows.append(xs[s].index_select(0, torch.div(order[a:b], L.k, rounding_mode="floor")))
            lids.append(local[a:b])
            src.append(b - a)
        y = L.experts(torch.cat(rows), torch.cat(lids))
        o = 0
        for s in range(W):
            y_parts[s][d] = y[o:o + src[s]]
            o += src[s]
    outs = []
    for s, L in enumerate(ranks):
        order = plans[s][0]
        n = xs[s].shape[0]
        y_back = torch.cat(y_parts[s])
        y = torch.empty_like(y_back)
        y[order] = y_back
        outs.append(L.finish(xs[s], ws_[s], y.view(n, L.k, L.H)))
    return outs


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False
