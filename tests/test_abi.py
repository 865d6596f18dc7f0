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
