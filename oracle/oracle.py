"""ctypes front-end of the CPU oracle (oracle/moe_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. Only
tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this module;
the product package never does.

Restates llama.cpp's CPU MUL_MAT_ID path as reproduced in the reference at
patches/trace-hook/ggml-cpu.c:1483-1767 (type pairing at :250-339). See
moe_oracle.h for what is pinned (block formats vs gguf-py) and what is not.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, Q4_0, Q5_0, Q8_0, Q8_1, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 0, 1, 2, 6, 8, 9, 10, 11, 12, 13, 14, 15
WEIGHT_TYPES = [Q4_0, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K]
TYPE_NAMES = {Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K",
              Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K", F32: "F32"}
BLCK = {Q4_0: 32, Q5_0: 32, Q8_0: 32, Q8_1: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_K: 256}
TSIZE = {Q4_0: 18, Q5_0: 22, Q8_0: 34, Q8_1: 36, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_K: 292}
GLU_SWIGLU, GLU_GEGLU, GLU_SWIGLU_OAI, GLU_SWIGLU_CLAMP, GLU_PRODUCT = 0, 1, 2, 3, 4

_lib = None


def build(force=False):
    """Compile liboracle.so with the committed Makefile."""
    src = os.path.join(HERE, "moe_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
        L.orc_row_size.restype = sz
        L.orc_row_size.argtypes = [i32, i64]
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.orc_fp16_to_fp32.restype = ctypes.c_float
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_dequantize_row.argtypes = [i32, vp, vp, i64]
        L.orc_quantize_row.argtypes = [i32, vp, vp, i64]
        L.orc_quantize_act.argtypes = [i32, vp, vp, i64]
        L.orc_vec_dot.argtypes = [i32, i32, i32, i64, vp, vp, vp]
        L.orc_mul_mat_id.argtypes = [i32, i32, i32, vp, i64, i64, i64, sz, vp, i64, i64, vp, i64, vp, i32]
        L.orc_mul_mat_id_q8_1.argtypes = [i32, vp, i64, i64, i64, sz, vp, i64, i64, vp, i64, vp, i32]
        L.orc_glu.restype = ctypes.c_float
        L.orc_glu.argtypes = [i32, ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.orc_topk_softmax.argtypes = [vp, i64, i64, i64, i32, vp, vp]
        L.orc_moe_layer.argtypes = [vp, vp, vp, i64, i32, i32, vp, vp, vp, i32]
        L.orc_fill_quantized.argtypes = [i32, vp, i64, i64, i64, ctypes.c_uint64, ctypes.c_float, i32]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def row_size(t, n):
    return (n // BLCK[t]) * TSIZE[t]


def vec_dot_type(t):
    return Q8_0 if t in (Q4_0, Q5_0, Q8_0) else Q8_K


def quantize(t, x):
    """f32 [..., n] -> uint8 [..., row_size] (weight quantizer)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.zeros(x.shape[:-1] + (row_size(t, n),), dtype=np.uint8)
    rc = lib().orc_quantize_row(t, _p(x), _p(out), x.size)
    assert rc == 0
    return out


def fill_quantized(t, out, row0, n_rows, n_cols, seed, sigma=0.02, n_threads=None):
    """Synthetic N(0, sigma) weights quantized to type t into `out` (uint8, n_rows rows)."""
    n_threads = n_threads or os.cpu_count() or 1
    assert out.flags.c_contiguous and out.nbytes >= n_rows * row_size(t, n_cols)
    rc = lib().orc_fill_quantized(t, _p(out), row0, n_rows, n_cols, seed, sigma, n_threads)
    assert rc == 0


def dequantize(t, q, n):
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows = q.size // row_size(t, n)
    out = np.zeros((rows, n), dtype=np.float32)
    rc = lib().orc_dequantize_row(t, _p(q), _p(out), rows * n)
    assert rc == 0
    return out


def quantize_act(t, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.zeros(x.shape[:-1] + (row_size(t, n),), dtype=np.uint8)
    rc = lib().orc_quantize_act(t, _p(x), _p(out), x.size)
    assert rc == 0
    return out


def vec_dot(t, act_t, exact, w_row, a_row, n):
    out = np.zeros(1, dtype=np.float32)
    w_row = np.ascontiguousarray(w_row, dtype=np.uint8)
    a_row = np.ascontiguousarray(a_row, dtype=np.uint8)
    rc = lib().orc_vec_dot(t, act_t, exact, n, _p(w_row), _p(a_row), _p(out))
    assert rc == 0
    return float(out[0])


def expert_ptrs(w):
    """uint8 [E][rows][row_bytes] -> array of per-expert pointers."""
    E = w.shape[0]
    base = w.ctypes.data
    stride = w.strides[0]
    return (ctypes.c_void_p * E)(*[base + e * stride for e in range(E)])


def mul_mat_id(t, w, K, src1, ids, act_t=None, exact=0, n_threads=8):
    """w uint8 [E][rows][row_bytes]; src1 f32 [n_tok][ne11][K]; ids i32 [n_tok][n_used]
    -> dst f32 [n_tok][n_used][rows]."""
    w = np.ascontiguousarray(w)
    src1 = np.ascontiguousarray(src1, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    E, rows = w.shape[0], w.shape[1]
    n_tok, ne11 = src1.shape[0], src1.shape[1]
    n_used = ids.shape[1]
    dst = np.zeros((n_tok, n_used, rows), dtype=np.float32)
    act_t = vec_dot_type(t) if act_t is None else act_t
    ptrs = expert_ptrs(w)
    rc = lib().orc_mul_mat_id(t, act_t, exact, ptrs, E, K, rows, row_size(t, K), _p(src1), ne11, n_tok,
                              _p(ids), n_used, _p(dst), n_threads)
    assert rc == 0, rc
    return dst


def mul_mat_id_q8_1(t, w, K, src1_q8_1, ids, n_threads=8):
    """Exact dots against an already-quantized Q8_1 src1 uint8 [n_tok][ne11][K/32*36]."""
    w = np.ascontiguousarray(w)
    src1_q8_1 = np.ascontiguousarray(src1_q8_1, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    E, rows = w.shape[0], w.shape[1]
    n_tok, ne11 = src1_q8_1.shape[0], src1_q8_1.shape[1]
    n_used = ids.shape[1]
    dst = np.zeros((n_tok, n_used, rows), dtype=np.float32)
    ptrs = expert_ptrs(w)
    rc = lib().orc_mul_mat_id_q8_1(t, ptrs, E, K, rows, row_size(t, K), _p(src1_q8_1), ne11, n_tok,
                                   _p(ids), n_used, _p(dst), n_threads)
    assert rc == 0, rc
    return dst


def glu(op, gate, up, limit=0.0):
    f = lib().orc_glu
    g = np.asarray(gate, dtype=np.float32).ravel()
    u = np.asarray(up, dtype=np.float32).ravel()
    out = np.array([f(op, float(a), float(b), float(limit)) for a, b in zip(g, u)], dtype=np.float32)
    return out.reshape(np.shape(gate))


def topk_softmax(logits, k, norm_w=False):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n_tok, E = logits.shape
    ids = np.zeros((n_tok, k), dtype=np.int32)
    w = np.zeros((n_tok, k), dtype=np.float32)
    rc = lib().orc_topk_softmax(_p(logits), n_tok, E, k, int(norm_w), _p(ids), _p(w))
    assert rc == 0
    return ids, w


class _Layer(ctypes.Structure):
    _fields_ = [("type_gate", ctypes.c_int), ("type_up", ctypes.c_int), ("type_down", ctypes.c_int),
                ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("shared_type", ctypes.c_int),
                ("shared_gate", ctypes.c_void_p), ("shared_up", ctypes.c_void_p), ("shared_down", ctypes.c_void_p),
                ("H", ctypes.c_int64), ("F", ctypes.c_int64), ("n_experts", ctypes.c_int64), ("k", ctypes.c_int64),
                ("glu_op", ctypes.c_int), ("glu_limit", ctypes.c_float), ("norm_w", ctypes.c_int)]


def moe_layer(layer, x, logits, act_mode=0, exact=0, n_threads=8):
    """layer: dict with types/weights (see tests/moe_data.py). x f32 [n_tok][H], logits f32 [n_tok][E].
    Returns (out [n_tok][H], ids, weights)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n_tok = x.shape[0]
    H, F, E, k = layer["H"], layer["F"], layer["E"], layer["k"]
    keep = []
    pg = expert_ptrs(layer["gate"]); pu = expert_ptrs(layer["up"]); pd = expert_ptrs(layer["down"])
    keep += [pg, pu, pd]
    L = _Layer()
    L.type_gate, L.type_up, L.type_down = layer["type_gate"], layer["type_up"], layer["type_down"]
    L.gate = ctypes.cast(pg, ctypes.c_void_p)
    L.up = ctypes.cast(pu, ctypes.c_void_p)
    L.down = ctypes.cast(pd, ctypes.c_void_p)
    if layer.get("shared_gate") is not None:
        L.shared_type = layer["shared_type"]
        L.shared_gate = layer["shared_gate"].ctypes.data
        L.shared_up = layer["shared_up"].ctypes.data
        L.shared_down = layer["shared_down"].ctypes.data
    else:
        L.shared_type = -1
    L.H, L.F, L.n_experts, L.k = H, F, E, k
    L.glu_op = layer.get("glu_op", GLU_SWIGLU)
    L.glu_limit = layer.get("glu_limit", 0.0)
    L.norm_w = int(layer.get("norm_w", False))
    out = np.zeros((n_tok, H), dtype=np.float32)
    ids = np.zeros((n_tok, k), dtype=np.int32)
    w = np.zeros((n_tok, k), dtype=np.float32)
    rc = lib().orc_moe_layer(ctypes.byref(L), _p(x), _p(logits), n_tok, act_mode, exact, _p(out), _p(ids), _p(w),
                             n_threads)
    assert rc == 0, rc
    return out, ids, w
