// moe-cache.cuh -- the hot-expert MoE path as llama.cpp's CUDA backend calls
// it (C++ linkage, ggml types). It declares the six functions whose names,
// arguments and meaning the backend's patched call sites use (kernels/
// moe-cache.cuh:15-40 of Zapdev-labs/a6000-custom-kernels); moe-cache.cu
// implements them on top of libmoe_b200.so's C ABI (moe_cache_b200.h).
// Drop both files into ggml/src/ggml-cuda/ of a llama.cpp tree (see
// apply_patches.py next to them).
#pragma once

#include "common.cuh"

#include <cstddef>

// GGML_CUDA_MOE_CACHE=1 turns the path on (read once).
bool ggml_cuda_moe_cache_enabled();

// Should this expert tensor (src0 of a MUL_MAT_ID) take the path?
bool ggml_cuda_moe_cache_wants(const ggml_tensor * src0);

// The MUL_MAT_ID decode GEMV through the expert pointer table, with the MMVQ
// fusion arguments (gate + GLU, biases, shared expert).
void ggml_cuda_moe_cache_mul_mat_vec_q(
        ggml_backend_cuda_context & ctx,
        const ggml_tensor * src0, const ggml_tensor * ids, ggml_tensor * dst,
        const ggml_cuda_mm_fusion_args_host * fusion, const ggml_cuda_mm_fusion_args_device & fusion_dev,
        const char * src1_q8_1, const int32_t * ids_d, float * dst_d,
        int64_t ne00, int64_t ne01, int64_t ne02, int64_t ne03,
        int64_t ncols_dst, int64_t s01, int64_t s02, int64_t s03,
        int64_t nchannels_y, int64_t nchannels_dst,
        int64_t stride_col_y, int64_t stride_col_dst,
        int64_t stride_channel_y, int64_t stride_channel_dst,
        int64_t ids_stride, cudaStream_t stream);

// Promotion pass between graph computes. With libmoe_b200 it only enqueues
// device work on `stream`.
void ggml_cuda_moe_cache_step(cudaStream_t stream);

// True once at least one tensor went through the path.
bool ggml_cuda_moe_cache_active();

// Make a host tensor GPU-readable (zero-copy); true when it is afterwards.
bool ggml_cuda_moe_cache_pin_host(const ggml_tensor * t);
