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
