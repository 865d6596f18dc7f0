"""Loader and ctypes declarations for libmoe_b200.so (the C ABI in include/moe_cache_b200.h).

The library is built in-tree by csrc/Makefile (nvcc, sm_100a). There is no
fallback: if the library cannot be built or loaded, every call raises.
"""
import ctypes
import os
import subprocess
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libmoe_b200.so")
REPO = os.path.dirname(PKG_DIR)
HEADER = os.path.join(REPO, "include", "moe_cache_b200.h")

MOE_OK, MOE_ERR_INVALID, MOE_ERR_UNSUPPORTED, MOE_ERR_CUDA, MOE_ERR_OOM, MOE_ERR_DEVICE, MOE_ERR_STATE = \
    0, -1, -2, -3, -4, -5, -6

_lock = threading.Lock()
_lib = None


class MoeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"moe_b200 error {code}: {msg}")
        self.code = code


class MoeTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("type", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_uint64 * 4), ("name", ctypes.c_char_p)]


class MoeFusionHost(ctypes.Structure):
    _fields_ = [("gate", ctypes.POINTER(MoeTensor))]


class MoeFusionDevice(ctypes.Structure):
    _fields_ = [("gate", ctypes.c_void_p), ("x_bias", ctypes.c_void_p), ("gate_bias", ctypes.c_void_p),
                ("x_scale", ctypes.c_void_p), ("gate_scale", ctypes.c_void_p), ("glu_op", ctypes.c_int32),
                ("glu_limit", ctypes.c_float), ("shared_up", ctypes.c_void_p), ("shared_gate", ctypes.c_void_p),
                ("shared_dst", ctypes.c_void_p), ("shared_stride_col_dst", ctypes.c_int64)]


class MoeCacheConfig(ctypes.Structure):
    _fields_ = [("enabled", ctypes.c_int32), ("slots", ctypes.c_int32), ("budget_gb", ctypes.c_double),
                ("seed_path", ctypes.c_char_p), ("claim_device", ctypes.c_int32), ("debug", ctypes.c_int32)]


class MoeCacheStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("steps", "hits", "misses", "promotions", "evictions", "resident",
                                               "registered", "log_overflow", "pool_bytes")]


class MoeLayerDesc(ctypes.Structure):
    _fields_ = [("gate", MoeTensor), ("up", MoeTensor), ("down", MoeTensor), ("shared_type", ctypes.c_int32),
                ("shared_gate", ctypes.c_void_p), ("shared_up", ctypes.c_void_p), ("shared_down", ctypes.c_void_p),
                ("H", ctypes.c_int64), ("F", ctypes.c_int64), ("n_experts", ctypes.c_int64), ("k", ctypes.c_int64),
                ("glu_op", ctypes.c_int32), ("glu_limit", ctypes.c_float), ("norm_w", ctypes.c_int32)]


def _sources():
    out = []
    for d in (CSRC, os.path.join(REPO, "include")):
        for f in os.listdir(d):
            if f.endswith((".cu", ".cuh", ".h", "Makefile")) or f == "Makefile":
                out.append(os.path.join(d, f))
    return out


def build(force=False):
    """Compile libmoe_b200.so for sm_100a with csrc/Makefile (nvcc)."""
    stale = force or not os.path.exists(LIB_PATH) or \
        os.path.getmtime(LIB_PATH) < max(os.path.getmtime(p) for p in _sources())
    if stale:
        subprocess.check_call(["make", "-s", "-j4", "-C", CSRC])
    return LIB_PATH


def _declare(L):
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    PT = ctypes.POINTER(MoeTensor)
    sigs = {
        "ggml_cuda_moe_cache_enabled": (i32, []),
        "ggml_cuda_moe_cache_wants": (i32, [PT]),
        "ggml_cuda_moe_cache_mul_mat_vec_q": (i32, [PT, ctypes.POINTER(MoeFusionHost), ctypes.POINTER(MoeFusionDevice),
                                                    vp, i32, vp, vp] + [i64] * 15 + [vp]),
        "ggml_cuda_moe_cache_step": (i32, [vp]),
        "ggml_cuda_moe_cache_active": (i32, []),
        "ggml_cuda_moe_cache_pin_host": (i32, [PT]),
        "moe_b200_configure": (i32, [ctypes.POINTER(MoeCacheConfig)]),
        "moe_b200_reset": (i32, []),
        "moe_b200_stats": (i32, [ctypes.POINTER(MoeCacheStats)]),
        "moe_b200_table": (i32, [vp, vp, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)]),
        "moe_b200_device_error": (i32, [vp, ctypes.POINTER(i32)]),
        "moe_b200_last_error": (ctypes.c_char_p, []),
        "moe_b200_quantize_act": (i32, [i32, vp, vp, i64, i64, vp]),
        "moe_b200_topk_softmax": (i32, [vp, i64, i64, i64, i32, vp, vp, vp]),
        "moe_b200_layer_workspace_size": (sz, [ctypes.POINTER(MoeLayerDesc), i64]),
        "moe_b200_layer_decode": (i32, [ctypes.POINTER(MoeLayerDesc), vp, vp, vp, i64, vp, sz, vp]),
        "moe_b200_fill_quantized": (i32, [i32, vp, i64, i64, ctypes.c_uint64, ctypes.c_float, vp]),
        "moe_b200_layer_decode_noalloc": (i32, [ctypes.POINTER(MoeLayerDesc), vp, vp, vp, i64, vp]),
        "moe_b200_noalloc_device_error": (i32, [vp, ctypes.POINTER(i32)]),
        "moe_b200_layer_fused": (i32, [ctypes.POINTER(MoeLayerDesc), i64]),
        "moe_b200_layer_set_fused": (i32, [i32]),
        "moe_b200_ep_layer_decode": (i32, [ctypes.POINTER(MoeLayerDesc), i64, i64, i32, vp, vp, vp, i64, vp, sz, vp]),
        "moe_b200_prefill_workspace_size": (sz, [ctypes.POINTER(MoeTensor), i64, i64]),
        "moe_b200_layer_prefill_workspace_size": (sz, [ctypes.POINTER(MoeLayerDesc), i64]),
        "moe_b200_layer_prefill": (i32, [ctypes.POINTER(MoeLayerDesc), vp, vp, vp, i64, vp, sz, vp]),
        "moe_b200_experts_prefill_workspace_size": (sz, [ctypes.POINTER(MoeLayerDesc), i64, i64]),
        "moe_b200_experts_prefill": (i32, [ctypes.POINTER(MoeLayerDesc), vp, i32, vp, i64, i64, vp, vp, sz, vp]),
        "moe_b200_shared_prefill": (i32, [ctypes.POINTER(MoeLayerDesc), vp, i64, vp, vp, sz, vp]),
        "moe_b200_combine": (i32, [vp, vp, vp, vp, i64, i64, i64, vp]),
        "moe_b200_ipc_alloc": (i32, [sz, ctypes.POINTER(vp)]),
        "moe_b200_ipc_free": (i32, [vp]),
        "moe_b200_ipc_handle": (i32, [vp, vp]),
        "moe_b200_ipc_open": (i32, [vp, ctypes.POINTER(vp)]),
        "moe_b200_ipc_close": (i32, [vp]),
        "moe_b200_ep_dispatch": (i32, [vp, i32, i32, i64, vp, i64, i64, i64, vp, i64, vp, vp]),
        "moe_b200_ep_wait": (i32, [vp, ctypes.c_uint32, vp]),
        "moe_b200_set_wait_limits": (i32, [i64, i64]),
        "moe_b200_ep_decode_buffer_bytes": (sz, [i64, i64, i64, i32]),
        "moe_b200_stack_workspace_size": (sz, [ctypes.POINTER(MoeLayerDesc), i64]),
        "moe_b200_stack_prepare": (i32, [ctypes.POINTER(MoeLayerDesc), i64, vp, vp, vp, vp, vp, sz, vp]),
        "moe_b200_stack_run": (i32, [ctypes.POINTER(MoeLayerDesc), i64, vp, sz, vp]),
        "moe_b200_ep_layer_decode_p2p": (i32, [ctypes.POINTER(MoeLayerDesc), i64, i64, vp, i32, i32, vp, vp, vp, vp,
                                               sz, vp]),
        "moe_b200_ep_experts_rows_workspace_size": (sz, [ctypes.POINTER(MoeLayerDesc), i64]),
        "moe_b200_ep_experts_rows": (i32, [ctypes.POINTER(MoeLayerDesc), vp, vp, i64, vp, vp, vp, vp, sz, vp]),
        "moe_b200_ep_return": (i32, [vp, i32, i64, vp, vp, vp, i64, vp, vp]),
        "moe_b200_prefill_mul_mat_id": (i32, [ctypes.POINTER(MoeTensor), vp, i64, vp, i64, i64, vp, vp, sz,
                                             ctypes.POINTER(i32), vp]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def lib():
    """The loaded C library (built on first use if missing or stale)."""
    global _lib
    with _lock:
        if _lib is None:
            build()
            _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def check(rc):
    if rc != MOE_OK:
        raise MoeError(rc, lib().moe_b200_last_error().decode(errors="replace"))
    return rc


def header_functions():
    """Names of the functions declared in include/moe_cache_b200.h."""
    import re
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)) -
                  {"sizeof", "if", "for", "while", "return"})
