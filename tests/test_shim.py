"""The llama.cpp adapter (a6000-custom-kernels_b200/shim/): it compiles
against the ggml declarations it uses (a stand-in header with just those),
links against libmoe_b200.so, exports the six C++ entry points the patched
backend calls, and answers through the C ABI; the patch script places its
hooks at the upstream anchors, refuses trees without them, and leaves a
patched tree alone."""
import os
import shutil
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "a6000-custom-kernels_b200")
SHIM = os.path.join(PKG, "shim")
STUB = os.path.join(REPO, "tests", "shim_stub")
CUDA = "/usr/local/cuda"

ENTRY = ("ggml_cuda_moe_cache_enabled", "ggml_cuda_moe_cache_wants", "ggml_cuda_moe_cache_mul_mat_vec_q",
         "ggml_cuda_moe_cache_step", "ggml_cuda_moe_cache_active", "ggml_cuda_moe_cache_pin_host")


@pytest.fixture(scope="module")
def shim_lib(tmp_path_factory, pkg):
    from importlib import import_module
    import_module("a6000-custom-kernels_b200._lib").build()
    d = tmp_path_factory.mktemp("shim")
    obj, so = str(d / "moe-cache.o"), str(d / "libshim.so")
    subprocess.check_call(["nvcc", "-std=c++17", "-O2", "-Xcompiler", "-fPIC", "-I", STUB, "-I",
                           os.path.join(REPO, "include"), "-c", os.path.join(SHIM, "moe-cache.cu"), "-o", obj])
    subprocess.check_call(["g++", "-shared", "-o", so, obj, "-L", PKG, "-lmoe_b200", f"-Wl,-rpath,{PKG}",
                           "-L", f"{CUDA}/lib64", "-lcudart"])
    return d, so


def test_adapter_exports_the_backend_entry_points(shim_lib):
    d, so = shim_lib
    out = subprocess.check_output(["nm", "-DC", "--defined-only", so], text=True)
    for name in ENTRY:
        assert f"{name}(" in out, name          # C++ (mangled) definitions, as the backend declares them
    undefined = subprocess.check_output(["nm", "-D", "--undefined-only", so], text=True)
    for name in ENTRY:
        assert name in undefined                # each calls the C symbol of the same name in libmoe_b200


def test_adapter_calls_through(shim_lib, tmp_path):
    d, so = shim_lib
    main = tmp_path / "main.cpp"
    main.write_text('''
#include "moe-cache.cuh"
#include <cstring>
int main() {
    ggml_tensor t;
    std::memset(&t, 0, sizeof(t));
    t.type = GGML_TYPE_Q2_K;                  // no buffer: never claimed
    t.ne[0] = 256; t.ne[1] = 4; t.ne[2] = 8; t.ne[3] = 1;
    std::printf("%d %d %d\\n", (int) ggml_cuda_moe_cache_enabled(), (int) ggml_cuda_moe_cache_wants(&t),
                (int) ggml_cuda_moe_cache_active());
    return 0;
}
''')
    exe = str(tmp_path / "main")
    subprocess.check_call(["g++", "-std=c++17", "-I", SHIM, "-I", STUB, "-I", f"{CUDA}/include", str(main), "-o", exe,
                           so, f"-Wl,-rpath,{os.path.dirname(so)}:{PKG}", "-L", f"{CUDA}/lib64", "-lcudart"])
    env = dict(os.environ, GGML_CUDA_MOE_CACHE="1")
    assert subprocess.check_output([exe], env=env, text=True).split() == ["1", "0", "0"]
    env["GGML_CUDA_MOE_CACHE"] = "0"
    assert subprocess.check_output([exe], env=env, text=True).split() == ["0", "0", "0"]


def _fake_tree(root):
    """Files of a llama.cpp tree holding the anchor lines (and some filler)."""
    cu = root / "ggml" / "src" / "ggml-cuda"
    cu.mkdir(parents=True)
    (cu / "mmvq.cu").write_text('#include "mmvq.cuh"\n#include "quantize.cuh"\n\nvoid f() {\n'
                                "    const int64_t ids_stride = ids ? ids->nb[1] / ggml_type_size(ids->type) : 0;\n"
                                "\n    mul_mat_vec_q_switch_type();\n}\n")
    (cu / "ggml-cuda.cu").write_text(
        '#include "ggml-cuda/common.cuh"\n\n'
        "static bool ggml_backend_cuda_device_offload_op(ggml_backend_dev_t dev, const ggml_tensor * op) {\n"
        "    return false;\n}\n\n"
        "static bool ggml_backend_cuda_device_supports_buft(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft) {\n"
        "    return false;\n}\n\nvoid g() {\n"
        "    ggml_cuda_graph_evaluate_and_capture(cuda_ctx, cgraph, use_cuda_graph, cuda_graph_update_required, graph_key);\n"
        "\n    return GGML_STATUS_SUCCESS;\n}\n")
    (cu / "CMakeLists.txt").write_text("add_library(ggml-cuda)\n")
    return cu


def test_patch_script(tmp_path):
    sys.path.insert(0, SHIM)
    import apply_patches as ap
    cu = _fake_tree(tmp_path)
    assert ap.main([str(tmp_path)]) == 0
    mmvq, core, cm = ((cu / n).read_text() for n in ("mmvq.cu", "ggml-cuda.cu", "CMakeLists.txt"))
    assert '#include "moe-cache.cuh"' in mmvq and "ggml_cuda_moe_cache_mul_mat_vec_q(ctx, src0" in mmvq
    assert mmvq.index("ggml_cuda_moe_cache_wants") < mmvq.index("mul_mat_vec_q_switch_type")
    assert core.count("ggml_cuda_moe_cache_enabled()") == 2 and "ggml_cuda_moe_cache_step(cuda_ctx->stream())" in core
    assert core.index("ggml_cuda_moe_cache_step") < core.index("return GGML_STATUS_SUCCESS")
    assert "target_link_libraries(ggml-cuda PRIVATE" in cm and "libmoe_b200.so" in cm
    assert (cu / "moe-cache.cu").exists() and (cu / "moe-cache.cuh").exists()
    before = {n: (cu / n).read_text() for n in ("mmvq.cu", "ggml-cuda.cu", "CMakeLists.txt")}
    assert ap.main([str(tmp_path)]) == 0                     # a patched tree is left alone
    assert before == {n: (cu / n).read_text() for n in before}
    other = tmp_path / "other"
    cu2 = _fake_tree(other)
    (cu2 / "ggml-cuda.cu").write_text('#include "ggml-cuda/common.cuh"\n')   # anchors missing
    snapshot = (cu2 / "mmvq.cu").read_text()
    assert ap.main([str(other)]) == 1
    assert (cu2 / "mmvq.cu").read_text() == snapshot                    # nothing written
