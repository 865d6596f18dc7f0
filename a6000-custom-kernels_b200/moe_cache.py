"""Python mirror of the reference's hot-expert-cache interface.

Same names, argument meaning and error behaviour as kernels/moe-cache.cuh:15-40
(ggml_cuda_moe_cache_enabled / wants / mul_mat_vec_q / step / active /
pin_host), over the C ABI of libmoe_b200.so. Device memory and streams come
from torch (plumbing only); every computation runs in the sm_100a library.
Errors raise MoeError instead of aborting the process.
"""
import ctypes

import torch

from ._lib import (MoeCacheConfig, MoeCacheStats, MoeFusionDevice, MoeFusionHost, MoeTensor, MoeError, check, lib)

# ggml_type ids
F32, Q4_0, Q5_0, Q8_0, Q8_1, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 0, 2, 6, 8, 9, 10, 11, 12, 13, 14, 15
WEIGHT_TYPES = (Q4_0, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K)
BLCK = {Q4_0: 32, Q5_0: 32, Q8_0: 32, Q8_1: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_K: 256}
TSIZE = {Q4_0: 18, Q5_0: 22, Q8_0: 34, Q8_1: 36, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_K: 292}
GLU_SWIGLU, GLU_GEGLU, GLU_SWIGLU_OAI, GLU_SWIGLU_CLAMP, GLU_PRODUCT = 0, 1, 2, 3, 4
TENSOR_VIEW, TENSOR_NO_BUFFER = 1, 2


def row_size(t, n):
    return (n // BLCK[t]) * TSIZE[t]


def _stream(stream):
    if stream is None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, torch.cuda.Stream):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def expert_tensor(buf, ggml_type, K, rows, name="", flags=0):
    """Descriptor of an expert weight tensor held in `buf` (uint8, [E][rows][row_bytes],
    contiguous; device or pinned host). ggml shape: ne = [K, rows, E, 1]."""
    E = buf.shape[0]
    rb = row_size(ggml_type, K)
    assert buf.shape[1] == rows and buf.shape[2] == rb and buf.is_contiguous()
    d = MoeTensor()
    d.data = buf.data_ptr()
    d.type = ggml_type
    d.flags = flags
    d.ne[0], d.ne[1], d.ne[2], d.ne[3] = K, rows, E, 1
    d.nb[0], d.nb[1], d.nb[2], d.nb[3] = TSIZE[ggml_type], rb, rb * rows, rb * rows * E
    d.name = name.encode() if name else b""
    d._keep = buf          # keep the storage alive with the descriptor
    return d


def enabled():
    """ggml_cuda_moe_cache_enabled (moe-cache.cu:345-363)."""
    return bool(lib().ggml_cuda_moe_cache_enabled())


def wants(src0):
    """ggml_cuda_moe_cache_wants (moe-cache.cu:442-469)."""
    return bool(lib().ggml_cuda_moe_cache_wants(ctypes.byref(src0)))


def active():
    """ggml_cuda_moe_cache_active (moe-cache.cu:365-368)."""
    return bool(lib().ggml_cuda_moe_cache_active())


def pin_host(t):
    """ggml_cuda_moe_cache_pin_host (moe-cache.cu:372-405)."""
    return bool(lib().ggml_cuda_moe_cache_pin_host(ctypes.byref(t)))


def step(stream=None):
    """ggml_cuda_moe_cache_step (moe-cache.cu:669-775): promotion between graphs."""
    check(lib().ggml_cuda_moe_cache_step(_stream(stream)))


def fusion_device(gate=None, x_bias=None, gate_bias=None, glu_op=GLU_SWIGLU, glu_limit=0.0, shared_up=None,
                  shared_gate=None, shared_dst=None, shared_stride_col_dst=0):
    f = MoeFusionDevice()
    f.gate = _ptr(gate)
    f.x_bias = _ptr(x_bias)
    f.gate_bias = _ptr(gate_bias)
    f.glu_op = glu_op
    f.glu_limit = glu_limit
    f.shared_up = _ptr(shared_up)
    f.shared_gate = _ptr(shared_gate)
    f.shared_dst = _ptr(shared_dst)
    f.shared_stride_col_dst = shared_stride_col_dst
    return f


def mul_mat_vec_q(src0, src1, src1_type, ids, dst, *, ncols_dst, nchannels_y, nchannels_dst, stride_col_y,
                  stride_col_dst, stride_channel_y, stride_channel_dst, ids_stride, fusion_gate=None,
                  fusion_dev=None, stream=None):
    """ggml_cuda_moe_cache_mul_mat_vec_q (moe-cache.cu:821-868) with the argument meaning of the reference.
    src1: Q8_1 blocks (src1_type=Q8_1, strides in blocks) or f32 (src1_type=F32, strides in floats)."""
    fh = MoeFusionHost()
    if fusion_gate is not None:
        fh.gate = ctypes.pointer(fusion_gate)
    fd = fusion_dev if fusion_dev is not None else None
    s01 = src0.nb[1] // TSIZE[src0.type]
    rc = lib().ggml_cuda_moe_cache_mul_mat_vec_q(
        ctypes.byref(src0), ctypes.byref(fh), ctypes.byref(fd) if fd is not None else None,
        _ptr(src1), src1_type, _ptr(ids), _ptr(dst),
        src0.ne[0], src0.ne[1], src0.ne[2], src0.ne[3],
        ncols_dst, s01, src0.nb[2] // TSIZE[src0.type], src0.nb[3] // TSIZE[src0.type],
        nchannels_y, nchannels_dst, stride_col_y, stride_col_dst, stride_channel_y, stride_channel_dst,
        ids_stride, _stream(stream))
    check(rc)


# ---- additions (no counterpart in the reference) ---------------------------

def configure(enabled=True, slots=320, budget_gb=30.0, seed_path=None, claim_device=True, debug=False):
    cfg = MoeCacheConfig()
    cfg.enabled = int(enabled)
    cfg.slots = slots
    cfg.budget_gb = budget_gb
    cfg.seed_path = seed_path.encode() if seed_path else None
    cfg.claim_device = int(claim_device)
    cfg.debug = int(debug)
    check(lib().moe_b200_configure(ctypes.byref(cfg)))


def reset():
    check(lib().moe_b200_reset())


def stats():
    s = MoeCacheStats()
    check(lib().moe_b200_stats(ctypes.byref(s)))
    return {n: getattr(s, n) for n, _ in MoeCacheStats._fields_}


def table(src0):
    """Decoded DEVICE table of a registered tensor: list of slot (>=0), -1 host, -2 direct."""
    n = src0.ne[2]
    out = (ctypes.c_int32 * n)()
    n_slots, tid = ctypes.c_int32(), ctypes.c_int32()
    check(lib().moe_b200_table(ctypes.c_void_p(src0.data), out, n, ctypes.byref(n_slots), ctypes.byref(tid)))
    return list(out), n_slots.value, tid.value


def device_error(stream=None):
    code = ctypes.c_int32()
    check(lib().moe_b200_device_error(_stream(stream), ctypes.byref(code)))
    return code.value


# device error codes (moe_b200_device_error)
DERR_BAD_ID, DERR_TIMEOUT_FULL, DERR_TIMEOUT_EMPTY, DERR_TIMEOUT_TAG, DERR_EP_OVERFLOW = 1, 3, 4, 8, 9


def set_wait_limits(kernel_wait_ns=0, exchange_wait_ns=0):
    """Limits of the bounded device waits (moe_b200_set_wait_limits); <= 0 restores the 2 s default."""
    check(lib().moe_b200_set_wait_limits(int(kernel_wait_ns), int(exchange_wait_ns)))


def quantize_act(act_type, x, stream=None):
    """f32 [rows, cols] (device) -> uint8 blocks [rows, row_size] (device), llama.cpp bit-exact."""
    assert x.dtype == torch.float32 and x.is_cuda and x.is_contiguous()
    rows, cols = x.shape
    y = torch.empty((rows, row_size(act_type, cols)), dtype=torch.uint8, device=x.device)
    check(lib().moe_b200_quantize_act(act_type, _ptr(x), _ptr(y), rows, cols, _stream(stream)))
    return y


def topk_softmax(logits, k, norm_w=False, stream=None):
    n_tok, E = logits.shape
    ids = torch.empty((n_tok, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((n_tok, k), dtype=torch.float32, device=logits.device)
    check(lib().moe_b200_topk_softmax(_ptr(logits), n_tok, E, k, int(norm_w), _ptr(ids), _ptr(w), _stream(stream)))
    return ids, w


def prefill_mul_mat_id(src0, x, ids, dst=None, workspace=None, stream=None):
    """Prefill MUL_MAT_ID (moe_b200_prefill_mul_mat_id): x f32 [n_tok, K] and
    ids i32 [n_tok, k] on the device -> dst f32 [n_tok, k, rows], llama.cpp CPU
    semantics. Returns (dst, used_tensor_cores)."""
    assert x.dtype == torch.float32 and x.is_cuda and x.is_contiguous() and ids.dtype == torch.int32
    n_tok, K = x.shape
    k = ids.shape[1]
    rows = src0.ne[1]
    if dst is None:
        dst = torch.empty((n_tok, k, rows), dtype=torch.float32, device=x.device)
    need = lib().moe_b200_prefill_workspace_size(ctypes.byref(src0), n_tok, k)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    used = ctypes.c_int32(0)
    check(lib().moe_b200_prefill_mul_mat_id(ctypes.byref(src0), _ptr(x), n_tok, _ptr(ids), k, ids.stride(0),
                                            _ptr(dst), _ptr(workspace), workspace.numel(), ctypes.byref(used),
                                            _stream(stream)))
    return dst, bool(used.value)


def set_layer_fused(mode):
    """Kernel of the layer decode (moe_b200_layer_set_fused): True / 1 the
    per-expert-group kernel (default), 2 the grid-exchange kernel, False / 0
    four launches."""
    check(lib().moe_b200_layer_set_fused(int(mode)))


def fill_quantized(ggml_type, dst, n_rows, n_cols, seed, sigma=0.02, stream=None):
    check(lib().moe_b200_fill_quantized(ggml_type, _ptr(dst), n_rows, n_cols, seed, sigma, _stream(stream)))


__all__ = ["MoeError", "MoeTensor", "enabled", "wants", "active", "pin_host", "step", "mul_mat_vec_q",
           "fusion_device", "expert_tensor", "configure", "reset", "stats", "table", "device_error",
           "quantize_act", "topk_softmax", "fill_quantized", "prefill_mul_mat_id", "set_wait_limits"]
