// moe_stack.cu -- planning and cooperative launch of the persistent stack
// kernel (moe_stack.cuh) for layers whose gate/up and down tensors share one
// type. The tile geometry is the per-expert-group kernel's (plan_layer2 at
// one token), so both cut rows the same way.
#include <cstdio>

#include "moe_aux.h"
#include "moe_stack.cuh"

namespace moe {

namespace {

constexpr int kStackSmemLimit = 227 * 1024;

template <int T>
cudaError_t launch_stack_t(const StackArgs &a, int grid, size_t smem, cudaStream_t st) {
    auto kern = moe_stack_kernel<T, T>;
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
    attr[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: the waits between CTAs end
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

bool stack_type_supported(int ta, int tb) {
    if (ta != tb) return false;
    switch (ta) {
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q6_K: case T_Q4_0: case T_Q5_0: case T_Q8_0: case T_Q5_K:
            return true;
        default:
            return false;
    }
}

int launch_stack(int type, StackArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    if (!stack_type_supported(type, type)) { *why = "no stack kernel for this type"; return -2; }
    // the geometry of the per-expert-group kernel at one token
    Layer2Args p{};
    p.gu = a.gu;
    p.dn = a.dn;
    p.n_tok = 1;
    p.k = a.k;
    p.n_experts = a.n_experts;
    p.timeout_ns = a.timeout_ns;
    int grid = 0;
    size_t smem = 0;
    const int rc = plan_layer2(type, type, p, &grid, &smem, why);
    if (rc) return rc;
    if (a.k > STACK_MAX_K) { *why = "the stack kernel handles k <= 32"; return -2; }
    a.gu = p.gu;
    a.dn = p.dn;
    a.n_rb = p.n_rb;
    a.stage_bytes = p.stage_bytes;
    a.act_bytes = p.act_bytes;
    a.timeout_ns = p.timeout_ns;
    // the routing buffers follow the layer kernel's control block; the ring
    // takes what is left. Every consumer warp takes tiles (the per-layer tile
    // counts are sized for 16 warps), and the ring should hold one layer of
    // this CTA's share so the next layer streams in behind the current one.
    a.route_off = p.ctrl_bytes;
    a.ctrl_bytes = (p.ctrl_bytes + static_cast<uint32_t>(sizeof(StackShared)) + 127u) & ~127u;
    const int64_t avail = kStackSmemLimit - static_cast<int64_t>(a.ctrl_bytes) - a.act_bytes;
    int fit = avail > 0 ? static_cast<int>(avail / a.stage_bytes) : 0;
    if (fit > GEMV_MAX_STAGES) fit = GEMV_MAX_STAGES;
    if (fit < 2) { *why = "activations and tiles do not fit in shared memory"; return -2; }
    const int nw = fit < GEMV_CONSUMER_WARPS ? fit : GEMV_CONSUMER_WARPS;
    a.n_tile_warps = nw;
    // A parity wait cannot tell phase p of a stage from phase p + 2. Tile g
    // of a stage follows tile g - S there; if g - S lies in an earlier phase
    // of the layer (gate/up or down), every consumer warp has passed it
    // behind a CTA barrier, so any warp may take g. Otherwise the warp that
    // took g - S must take g too: S a multiple of nw.
    const int nu = a.k + (a.has_shared ? 1 : 0);
    const int cmin = 1 + (grid - nu) / nu;                      // smallest CTA group
    const int max_a = ((a.gu.nrows + cmin - 1) / cmin + a.gu.rows_per_tile - 1) / a.gu.rows_per_tile;
    const int max_b = ((a.dn.nrows + cmin - 1) / cmin + a.dn.rows_per_tile - 1) / a.dn.rows_per_tile;
    a.n_stages = max_a <= fit && max_b <= fit ? fit : fit / nw * nw;
    a.gu.n_tile_warps = nw;
    a.dn.n_tile_warps = nw;
    smem = static_cast<size_t>(a.ctrl_bytes) + a.act_bytes + static_cast<size_t>(a.n_stages) * a.stage_bytes;
    cudaError_t e = cudaErrorInvalidValue;
    switch (type) {
        case T_Q2_K: e = launch_stack_t<T_Q2_K>(a, grid, smem, st); break;
        case T_Q3_K: e = launch_stack_t<T_Q3_K>(a, grid, smem, st); break;
        case T_Q4_K: e = launch_stack_t<T_Q4_K>(a, grid, smem, st); break;
        case T_Q6_K: e = launch_stack_t<T_Q6_K>(a, grid, smem, st); break;
        case T_Q4_0: e = launch_stack_t<T_Q4_0>(a, grid, smem, st); break;
        case T_Q5_0: e = launch_stack_t<T_Q5_0>(a, grid, smem, st); break;
        case T_Q8_0: e = launch_stack_t<T_Q8_0>(a, grid, smem, st); break;
        case T_Q5_K: e = launch_stack_t<T_Q5_K>(a, grid, smem, st); break;
        default: break;
    }
    if (e != cudaSuccess) { *cuda_err = e; *why = "stack kernel launch"; return -3; }
    return 0;
}

}  // namespace moe
