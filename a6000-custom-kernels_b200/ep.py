"""Expert parallelism for MoE decode.

Each rank holds a contiguous 1/world of every layer's experts (the reference's
cache is single-GPU; the partition follows the expert-major tensor layout, so a
rank's experts are one contiguous slice of each tensor). Every rank routes the
same tokens over ALL experts (replicated logits and activations: at decode
batch sizes that is a few KB), runs the GEMVs on the picks it holds
(moe_b200_ep_layer_decode), and the ranks sum their shares of the weighted
combine with one all-reduce (NCCL over NVLink on GPUs, gloo on CPU). The
shared expert runs on rank 0 only.
"""
import ctypes

import torch

from ._lib import MoeLayerDesc, check, lib
from .moe_cache import _ptr, _stream, expert_tensor


def expert_range(n_experts, rank, world):
    """Global experts [lo, hi) held by `rank` of `world` (contiguous, balanced)."""
    return n_experts * rank // world, n_experts * (rank + 1) // world


class EPMoELayer:
    """This rank's share of one MoE layer. Built from a full MoELayer (same
    weights as the single-GPU layer) by slicing its expert tensors; the full
    tensors are not kept."""

    def __init__(self, full, rank, world, group=None):
        self.H, self.F, self.E, self.k = full.H, full.F, full.E, full.k
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = expert_range(full.E, rank, world)
        self.device = full.device
        self.types = dict(full.types)
        shapes = {"gate": (full.F, full.H), "up": (full.F, full.H), "down": (full.H, full.F)}
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


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False
