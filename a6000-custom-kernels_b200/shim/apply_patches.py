#!/usr/bin/env python3
"""Wire libmoe_b200.so into a llama.cpp tree.

Targets the llama.cpp commit the reference patches (11fe0215): the same four
call sites as the reference's patch set (patches/apply_patches.py of
Zapdev-labs/a6000-custom-kernels) -- the MUL_MAT_ID decode intercept in
mmvq.cu, the offload gate and the buffer-type gate in ggml-cuda.cu, and the
promotion step after each graph compute -- plus the build lines that link
libmoe_b200.so. It also copies moe-cache.cu / moe-cache.cuh (this directory)
into ggml/src/ggml-cuda/.

Every hook goes right after one line of upstream source (its anchor). An
anchor that is missing or appears more than once stops the script before any
file is written; a file that already carries the hooks (it mentions
libmoe_b200) is left alone, so running the script twice is harmless.

    python apply_patches.py <llama.cpp dir> [--lib <path to libmoe_b200.so>] [--include <dir of moe_cache_b200.h>]
"""
import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
MARK = "libmoe_b200"

# (file relative to the tree, anchor line, lines inserted after it)
HOOKS = [
    ("ggml/src/ggml-cuda/mmvq.cu", '#include "mmvq.cuh"',
     ['#include "moe-cache.cuh"   // libmoe_b200']),
    ("ggml/src/ggml-cuda/mmvq.cu", "    const int64_t ids_stride = ids ? ids->nb[1] / ggml_type_size(ids->type) : 0;",
     ["",
      "    // libmoe_b200: MUL_MAT_ID decode of registered expert tensors through the expert pointer table",
      "    if (ids && ggml_cuda_moe_cache_wants(src0)) {",
      "        ggml_cuda_moe_cache_mul_mat_vec_q(ctx, src0, ids, dst, fusion, fusion_local, src1_q8_1.get(), ids_d,",
      "                                          dst_d, ne00, ne01, ne02, ne03, ncols_dst, s01, s02, s03, nchannels_y,",
      "                                          nchannels_dst, stride_col_y, stride_col_dst, stride_channel_y,",
      "                                          stride_channel_dst, ids_stride, stream);",
      "        return;",
      "    }"]),
    ("ggml/src/ggml-cuda/ggml-cuda.cu", '#include "ggml-cuda/common.cuh"',
     ['#include "ggml-cuda/moe-cache.cuh"   // libmoe_b200']),
    ("ggml/src/ggml-cuda/ggml-cuda.cu",
     "static bool ggml_backend_cuda_device_offload_op(ggml_backend_dev_t dev, const ggml_tensor * op) {",
     ["    // libmoe_b200: every MUL_MAT_ID runs on the GPU (decode through the expert table,",
      "    // prefill reading pinned host experts in place)",
      "    if (op->op == GGML_OP_MUL_MAT_ID && ggml_cuda_moe_cache_enabled()) {",
      "        return true;",
      "    }"]),
    ("ggml/src/ggml-cuda/ggml-cuda.cu",
     "static bool ggml_backend_cuda_device_supports_buft(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft) {",
     ["    // libmoe_b200: pinned host buffers are read in place (no VRAM copy of host-resident experts)",
      "    if (ggml_cuda_moe_cache_enabled() && ggml_backend_buft_is_cuda_host(buft)) {",
      "        return true;",
      "    }"]),
    ("ggml/src/ggml-cuda/ggml-cuda.cu",
     "    ggml_cuda_graph_evaluate_and_capture(cuda_ctx, cgraph, use_cuda_graph, cuda_graph_update_required, graph_key);",
     ["",
      "    // libmoe_b200: the cache's promotion step (device work on the stream, after capture ended)",
      "    if (ggml_cuda_moe_cache_active()) {",
      "        ggml_cuda_moe_cache_step(cuda_ctx->stream());",
      "    }"]),
]


def plan(tree, lib, include):
    """The new text of every file to change, or an error message."""
    edits = {}
    for rel, anchor, lines in HOOKS:
        path = os.path.join(tree, rel)
        if not os.path.exists(path):
            return None, f"{path}: missing"
        text = edits.get(rel, open(path).read())
        if MARK in open(path).read():
            continue
        hits = [i for i, l in enumerate(text.split("\n")) if l == anchor]
        if len(hits) != 1:
            return None, f"{path}: anchor found {len(hits)} times: {anchor.strip()}"
        rows = text.split("\n")
        rows[hits[0] + 1:hits[0] + 1] = lines
        edits[rel] = "\n".join(rows)
    cm = "ggml/src/ggml-cuda/CMakeLists.txt"
    path = os.path.join(tree, cm)
    if not os.path.exists(path):
        return None, f"{path}: missing"
    text = open(path).read()
    if MARK not in text:
        edits[cm] = text.rstrip("\n") + "\n\n# libmoe_b200: hot-expert MoE path for B200 (sm_100a)\n" + \
            f'target_include_directories(ggml-cuda PRIVATE "{include}")\n' + \
            f'target_link_libraries(ggml-cuda PRIVATE "{lib}")\n'
    return edits, None


def main(argv=None):
    ap = argparse.ArgumentParser(description="wire libmoe_b200.so into a llama.cpp tree")
    ap.add_argument("tree")
    ap.add_argument("--lib", default=os.path.join(PKG, "libmoe_b200.so"))
    ap.add_argument("--include", default=os.path.join(REPO, "include"))
    args = ap.parse_args(argv)
    edits, err = plan(args.tree, os.path.abspath(args.lib), os.path.abspath(args.include))
    if err:
        print(f"apply_patches: {err}; nothing written", file=sys.stderr)
        return 1
    dst = os.path.join(args.tree, "ggml/src/ggml-cuda")
    for name in ("moe-cache.cu", "moe-cache.cuh"):
        shutil.copyfile(os.path.join(HERE, name), os.path.join(dst, name))
    for rel, text in edits.items():
        with open(os.path.join(args.tree, rel), "w") as f:
            f.write(text)
        print(f"patched {rel}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
