"""The C-ABI library loads on a machine without a GPU and exports every
function include/moe_cache_b200.h declares (no compute calls here)."""
import ctypes
import subprocess

from conftest import REPO  # noqa: F401


def test_library_exports_header_symbols(pkg):
    L = pkg.lib()
    names = pkg._lib.header_functions()
    assert "ggml_cuda_moe_cache_mul_mat_vec_q" in names and len(names) >= 17
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", pkg._lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(names) <= exported


def test_reference_entry_points_present(pkg):
    for n in ("enabled", "wants", "mul_mat_vec_q", "step", "active", "pin_host"):
        assert hasattr(pkg._lib.lib(), "ggml_cuda_moe_cache_" + n)


def test_struct_layouts(pkg):
    from importlib import import_module
    lib_mod = import_module("a6000-custom-kernels_b200._lib")
    assert ctypes.sizeof(lib_mod.MoeTensor) == 8 + 4 + 4 + 32 + 32 + 8
    assert ctypes.sizeof(lib_mod.MoeFusionDevice) == 5 * 8 + 4 + 4 + 3 * 8 + 8


def test_env_and_config_without_gpu(pkg, monkeypatch):
    mc = pkg.moe_cache
    mc.reset()
    monkeypatch.setenv("GGML_CUDA_MOE_CACHE", "0")
    assert mc.enabled() is False
    mc.reset()
    monkeypatch.setenv("GGML_CUDA_MOE_CACHE", "1")
    assert mc.enabled() is True
    assert mc.active() is False
    mc.configure(enabled=False)
    assert mc.enabled() is False
    s = mc.stats()
    assert s["registered"] == 0 and s["steps"] == 0
    mc.reset()


def test_errors_are_status_codes_not_aborts(pkg):
    L = pkg.lib()
    rc = L.moe_b200_quantize_act(3, None, None, 1, 32, None)
    assert rc == pkg._lib.MOE_ERR_UNSUPPORTED
    assert b"act_type" in L.moe_b200_last_error()
    rc = L.moe_b200_topk_softmax(None, 1, 4, 8, 0, None, None, None)
    assert rc == pkg._lib.MOE_ERR_INVALID
    rc = L.moe_b200_prefill_mul_mat_id(None, None, 1, None, 8, 8, None, None, 0, None, None)
    assert rc == pkg._lib.MOE_ERR_INVALID
    assert L.moe_b200_prefill_workspace_size(None, 1, 8) == 0


def test_stack_prepare_rejects_unsupported_type_mixes(pkg):
    """The stack takes one type for every tensor of every layer, or per-layer
    types when gate = up and every type is among Q2_K, Q3_K, Q4_K, Q6_K; any
    other mix is refused with a status code before anything touches the GPU."""
    from importlib import import_module
    lm = import_module("a6000-custom-kernels_b200._lib")
    L = pkg.lib()
    H, F, E, k = 1024, 512, 16, 4

    def desc(tg, tu, td):
        d = lm.MoeLayerDesc()
        for name, t, (rows, K) in (("gate", tg, (F, H)), ("up", tu, (F, H)), ("down", td, (H, F))):
            m = getattr(d, name)
            m.data, m.type = 0x1000, t
            m.ne[0], m.ne[1], m.ne[2], m.ne[3] = K, rows, E, 1
        d.shared_type, d.H, d.F, d.n_experts, d.k = -1, H, F, E, k
        return d

    Q4_0, Q2_K, Q3_K = 2, 10, 11
    dummy = (ctypes.c_void_p * 2)(0x1000, 0x1000)
    for pair in ((desc(Q2_K, Q2_K, Q2_K), desc(Q4_0, Q4_0, Q4_0)),     # a legacy type in a mixed stack
                 (desc(Q2_K, Q2_K, Q3_K), desc(Q3_K, Q2_K, Q3_K))):    # gate and up of different types
        arr = (lm.MoeLayerDesc * 2)(*pair)
        need = L.moe_b200_stack_workspace_size(ctypes.byref(arr[0]), 2)
        ws = ctypes.create_string_buffer(need)
        rc = L.moe_b200_stack_prepare(arr, 2, dummy, dummy, dummy, None, ws, need, None)
        assert rc == lm.MOE_ERR_UNSUPPORTED, rc
        assert b"Q2_K, Q3_K, Q4_K, Q6_K" in L.moe_b200_last_error()
