// moe_layer_launch.cuh -- cooperative launch of one moe_layer_kernel
// instantiation (explicitly instantiated per gate/up type in moe_layer_*.cu).
#pragma once
#include <cstdio>

#include "moe_layer2.cuh"

namespace moe {

extern char g_layer_diag[256];

// One member per pass for every batch size: measured faster at 8 tokens than
// sharing the weight decode across 2, 4 or 8 members (those keep more
// registers live and spill), and the row split weighs groups by members.
template <int TA, int TB>
cudaError_t launch_layer_t(const LayerArgs &a, int grid, size_t smem, cudaStream_t st) {
    auto kern = moe_layer_kernel<TA, TB, 1>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    bool &done = configured[dev];
    if (!done) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident: one grid barrier
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        snprintf(g_layer_diag, sizeof(g_layer_diag), "grid=%d threads=%d smem=%zu regs=%d maxThreads=%d local=%zu",
                 grid, GEMV_THREADS, smem, fa.numRegs, fa.maxThreadsPerBlock, fa.localSizeBytes);
    }
    return e;
}

// The per-expert-group kernel (moe_layer2.cuh), same launch shape.
template <int TA, int TB>
cudaError_t launch_layer2_t(const Layer2Args &a, int grid, size_t smem, cudaStream_t st) {
    auto kern = moe_layer2_kernel<TA, TB>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident: the h waits inside a group end
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        snprintf(g_layer_diag, sizeof(g_layer_diag), "grid=%d threads=%d smem=%zu regs=%d local=%zu", grid,
                 GEMV_THREADS, smem, fa.numRegs, fa.localSizeBytes);
    }
    return e;
}

}  // namespace moe
