"""One MoE FFN layer on the B200 path: the graph around two MUL_MAT_ID calls.

Routing (top-k + softmax), the fused gate/up GEMV with the GLU and the shared
expert, the down GEMV and the weighted combine run as four sm_100a launches of
libmoe_b200.so (moe_b200_layer_decode). This mirrors what llama.cpp's graph does
around the reference's intercepted MUL_MAT_ID calls (build_moe_ffn order:
route, gate/up, GLU, down, weight, sum over picks, add the shared expert).
"""
import ctypes

import torch

from ._lib import MoeLayerDesc, check, lib
from .moe_cache import GLU_SWIGLU, _ptr, _stream, expert_tensor, fill_quantized, row_size


class MoELayer:
    """Expert weights live in `device` memory (HBM-resident) unless `host=True`,
    in which case they live in pinned host memory behind the tiered cache."""

    def __init__(self, H, F, n_experts, k, types, shared=True, glu_op=GLU_SWIGLU, glu_limit=0.0, norm_w=False,
                 device="cuda", host=False, name="blk.0", seed=0, weights=None, sigma=0.02):
        self.H, self.F, self.E, self.k = H, F, n_experts, k
        self.types = dict(types)          # {"gate": t, "up": t, "down": t}
        self.glu_op, self.glu_limit, self.norm_w = glu_op, glu_limit, norm_w
        self.device = torch.device(device)
        shapes = {"gate": (F, H), "up": (F, H), "down": (H, F)}
        self.w = {}
        for i, role in enumerate(("gate", "up", "down")):
            t = self.types[role]
            rows, K = shapes[role]
            if weights is not None:
                src = torch.as_tensor(weights[role])
                buf = src.pin_memory() if host else src.to(self.device)
            else:
                buf = torch.empty((n_experts, rows, row_size(t, K)), dtype=torch.uint8, device=self.device)
                fill_quantized(t, buf, n_experts * rows, K, seed * 1000003 + i, sigma=sigma)
                if host:
                    pinned = torch.empty(buf.shape, dtype=torch.uint8, pin_memory=True)
                    pinned.copy_(buf)
                    buf = pinned
            self.w[role] = buf
        self.desc_t = {r: expert_tensor(self.w[r], self.types[r], shapes[r][1], shapes[r][0],
                                        name=f"{name}.ffn_{r}_exps.weight") for r in ("gate", "up", "down")}
        self.shared = {}
        if shared:
            for i, role in enumerate(("gate", "up", "down")):
                t = self.types[role]
                rows, K = shapes[role]
                if weights is not None and weights.get(f"shared_{role}") is not None:
                    buf = torch.as_tensor(weights[f"shared_{role}"]).to(self.device)
                else:
                    buf = torch.empty((rows, row_size(t, K)), dtype=torch.uint8, device=self.device)
                    fill_quantized(t, buf, rows, K, seed * 1000003 + 7 + i, sigma=sigma)
                self.shared[role] = buf
        d = MoeLayerDesc()
        d.gate, d.up, d.down = self.desc_t["gate"], self.desc_t["up"], self.desc_t["down"]
        d.shared_type = self.types["up"] if shared else -1
        d.shared_gate = _ptr(self.shared.get("gate"))
        d.shared_up = _ptr(self.shared.get("up"))
        d.shared_down = _ptr(self.shared.get("down"))
        d.H, d.F, d.n_experts, d.k = H, F, n_experts, k
        d.glu_op, d.glu_limit, d.norm_w = glu_op, glu_limit, int(norm_w)
        self.desc = d
        self._ws = {}

    def weight_bytes_per_token(self):
        """Expert bytes one batch-1 token streams: k routed + shared experts x 3 matrices."""
        per = sum(self.w[r][0].numel() for r in ("gate", "up", "down"))
        return per * (self.k + (1 if self.shared else 0))

    def workspace(self, n_tok):
        ws = self._ws.get(n_tok)
        if ws is None:
            nbytes = lib().moe_b200_layer_workspace_size(ctypes.byref(self.desc), n_tok)
            # zero-filled once: the fused kernel's launch epoch lives at its start
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[n_tok] = ws
        return ws

    def fused(self, n_tok):
        """True when decode() runs the layer as one fused kernel for n_tok tokens."""
        return bool(lib().moe_b200_layer_fused(ctypes.byref(self.desc), n_tok))

    def decode(self, x, logits, out=None, stream=None, trace=None):
        """x f32 [n_tok, H], logits f32 [n_tok, E] (device) -> out f32 [n_tok, H].
        With `trace` (a seed.TraceWriter) the step's routing is appended as one
        record per expert tensor, as the reference's trace hook writes it for
        each MUL_MAT_ID (this reads the ids back to the host)."""
        n_tok = x.shape[0]
        if out is None:
            out = torch.empty((n_tok, self.H), dtype=torch.float32, device=self.device)
        ws = self.workspace(n_tok)
        check(lib().moe_b200_layer_decode(ctypes.byref(self.desc), _ptr(x), _ptr(logits), _ptr(out), n_tok,
                                          _ptr(ws), ws.numel(), _stream(stream)))
        if trace is not None:
            ids = self.routing_of(n_tok)[0].cpu().numpy()
            for r in ("gate", "up", "down"):
                trace.record(self.desc_t[r].name.decode(), ids, self.E)
        return out

    def prefill(self, x, logits, out=None, stream=None):
        """x f32 [n_tok, H], logits f32 [n_tok, E] (device) -> out f32 [n_tok, H] for any
        n_tok: the tensor-core prefill path (moe_b200_layer_prefill)."""
        n_tok = x.shape[0]
        if out is None:
            out = torch.empty((n_tok, self.H), dtype=torch.float32, device=self.device)
        key = ("prefill", n_tok)
        ws = self._ws.get(key)
        if ws is None:
            nbytes = lib().moe_b200_layer_prefill_workspace_size(ctypes.byref(self.desc), n_tok)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        check(lib().moe_b200_layer_prefill(ctypes.byref(self.desc), _ptr(x), _ptr(logits), _ptr(out), n_tok,
                                           _ptr(ws), ws.numel(), _stream(stream)))
        return out

    def prefill_intermediates(self, n_tok):
        """Views of the last prefill's workspace (layout of moe_b200_layer_prefill):
        ids [n][k], weights [n][k], gate [n][k][F], h [n][k][F] (GLU output),
        y [n][k][H] (down outputs), then with a shared expert its gate [n][F],
        hs [n][F] and ys [n][H]."""
        ws = self._ws[("prefill", n_tok)]
        n, k, F, H = n_tok, self.k, self.F, self.H
        parts = [(n * k, torch.int32, (n, k)), (n * k, torch.float32, (n, k)), (n * k * F, torch.float32, (n, k, F)),
                 (n * k * F, torch.float32, (n, k, F)), (n * k * H, torch.float32, (n, k, H))]
        if self.shared:
            parts += [(n * F, torch.float32, (n, F)), (n * F, torch.float32, (n, F)), (n * H, torch.float32, (n, H))]
        out, off = [], 0
        for count, dt, shape in parts:
            nbytes = 4 * count
            out.append(ws[off: off + nbytes].view(dt).view(shape))
            off += (nbytes + 255) // 256 * 256
        return tuple(out)

    def intermediates(self, n_tok):
        """Views of the last decode's workspace (layout of moe_b200_layer_decode):
        ids [n][k], weights [n][k], h [n][k][F] (GLU output), hs [n][F] (shared
        GLU output), y [n][k][H] (down outputs), ys [n][H] (shared down)."""
        ws = self._ws[n_tok]
        n, k, F, H = n_tok, self.k, self.F, self.H
        # the first 256 bytes hold the fused kernels' launch epoch, then the
        # per-expert-group kernel's row counters (8 tokens x H / 64 blocks)
        out, off = [], 256 + (4 * 8 * ((H + 63) // 64) + 255) // 256 * 256
        for count, dt, shape in ((n * k, torch.int32, (n, k)), (n * k, torch.float32, (n, k)),
                                 (n * k * F, torch.float32, (n, k, F)), (n * F, torch.float32, (n, F)),
                                 (n * k * H, torch.float32, (n, k, H)), (n * H, torch.float32, (n, H))):
            nbytes = 4 * count
            out.append(ws[off: off + nbytes].view(dt).view(shape))
            off += (nbytes + 255) // 256 * 256
        return tuple(out)

    def routing_of(self, n_tok):
        """(ids, weights) views of the last decode's routing in the workspace."""
        ids, w = self.intermediates(n_tok)[:2]
        return ids, w


class Stack:
    """Batch-1 layers decoded back to back in one persistent launch
    (moe_b200_stack_prepare / moe_b200_stack_run). Layer l reads xs[l] and
    logits[l] (device f32 [1, H] / [1, E]), writes outs[l] and, with
    x_nexts, x_nexts[l] = xs[l] + outs[l] (a residual chain when xs[l + 1]
    is x_nexts[l]). The layers share one shape; their types are either one
    type for every tensor or, per layer, gate = up with the gate/up and down
    types among Q2_K, Q3_K, Q4_K, Q6_K (the mixed-type kernel). run() may be
    repeated; every tensor must stay alive."""

    def __init__(self, layers, xs, logits, outs, x_nexts=None, stream=None):
        n = len(layers)
        self.layers, self.n = layers, n
        self.desc0 = layers[0].desc
        arr = (MoeLayerDesc * n)(*[L.desc for L in layers])
        nbytes = lib().moe_b200_stack_workspace_size(ctypes.byref(self.desc0), n)
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=layers[0].device)

        def ptrs(ts):
            return (ctypes.c_void_p * n)(*[_ptr(t) for t in ts])
        check(lib().moe_b200_stack_prepare(arr, n, ptrs(xs), ptrs(logits), ptrs(outs),
                                           ptrs(x_nexts) if x_nexts is not None else None, _ptr(self.ws),
                                           self.ws.numel(), _stream(stream)))

    def run(self, stream=None):
        check(lib().moe_b200_stack_run(ctypes.byref(self.desc0), self.n, _ptr(self.ws), self.ws.numel(),
                                       _stream(stream)))

