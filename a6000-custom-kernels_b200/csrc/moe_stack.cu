// moe_stack.cu -- planning and cooperative launch of the persistent stack
// kernel (moe_stack.cuh): for layers whose gate/up and down tensors share one
// type, and for mixed stacks whose layers pick their gate/up and down types
// among Q2_K, Q3_K, Q4_K and Q6_K. The tile geometry of each type is the
// per-expert-group kernel's (plan_layer2 at one token).
#include <algorithm>
#include <cstdio>

#include "moe_aux.h"
#include "moe_stack.cuh"

namespace moe {

namespace {

constexpr int kStackSmemLimit = 227 * 1024;
constexpr uint32_t kMixStageCap = 14 * 1024;   // mixed stacks: stage bytes to aim below

template <int T>
cudaError_t launch_stack_t(const StackArgs &a, int grid, size_t smem, cudaStream_t st) {
    auto kern = moe_stack_kernel<T, T>;   // T_STACK_MIXED: the mixed-type kernel
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

namespace {

// The ring for the geometry in a (gu / dn of every type in use): stages of
// a.stage_bytes in what shared memory is left after the control block, the
// routing buffers and the activations; max_a / max_b = the most tiles one CTA
// takes in a phase of any layer.
int fit_ring(StackArgs &a, int max_a, int max_b, const char **why) {
    const int64_t avail = kStackSmemLimit - static_cast<int64_t>(a.ctrl_bytes) - a.act_bytes;
    int fit = avail > 0 ? static_cast<int>(avail / a.stage_bytes) : 0;
    if (fit > GEMV_MAX_STAGES) fit = GEMV_MAX_STAGES;
    if (fit < 2) { *why = "activations and tiles do not fit in shared memory"; return -2; }
    // every consumer warp takes tiles (the per-layer tile counts are sized
    // for 16 warps), and the ring should hold one layer of this CTA's share
    // so the next layer streams in behind the current one
    const int nw = fit < GEMV_CONSUMER_WARPS ? fit : GEMV_CONSUMER_WARPS;
    a.n_tile_warps = nw;
    // A parity wait cannot tell phase p of a stage from phase p + 2. Tile g
    // of a stage follows tile g - S there; if g - S lies in an earlier phase
    // of the layer (gate/up or down), every consumer warp has passed it
    // behind a CTA barrier, so any warp may take g. Otherwise the warp that
    // took g - S must take g too: S a multiple of nw.
    a.n_stages = max_a <= fit && max_b <= fit ? fit : fit / nw * nw;
    return 0;
}

// bytes of one 256-value block of a mixed-stack type
int mix_block_bytes(int t) {
    switch (t) {
        case T_Q2_K: return fmt<T_Q2_K>::bytes;
        case T_Q3_K: return fmt<T_Q3_K>::bytes;
        case T_Q4_K: return fmt<T_Q4_K>::bytes;
        default: return fmt<T_Q6_K>::bytes;
    }
}

// the most tiles of rows / rpt rows one CTA takes (its group has at least cmin CTAs)
int max_tiles(int rows, int cmin, int rpt) { return ((rows + cmin - 1) / cmin + rpt - 1) / rpt; }

cudaError_t launch_by_type(int type, const StackArgs &a, int grid, size_t smem, cudaStream_t st) {
    switch (type) {
        case T_Q2_K: return launch_stack_t<T_Q2_K>(a, grid, smem, st);
        case T_Q3_K: return launch_stack_t<T_Q3_K>(a, grid, smem, st);
        case T_Q4_K: return launch_stack_t<T_Q4_K>(a, grid, smem, st);
        case T_Q6_K: return launch_stack_t<T_Q6_K>(a, grid, smem, st);
        case T_Q4_0: return launch_stack_t<T_Q4_0>(a, grid, smem, st);
        case T_Q5_0: return launch_stack_t<T_Q5_0>(a, grid, smem, st);
        case T_Q8_0: return launch_stack_t<T_Q8_0>(a, grid, smem, st);
        case T_Q5_K: return launch_stack_t<T_Q5_K>(a, grid, smem, st);
        case T_STACK_MIXED: return launch_stack_t<T_STACK_MIXED>(a, grid, smem, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

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
    // takes what is left
    a.route_off = p.ctrl_bytes;
    a.ctrl_bytes = (p.ctrl_bytes + static_cast<uint32_t>(sizeof(StackShared)) + 127u) & ~127u;
    const int nu = a.k + (a.has_shared ? 1 : 0);
    const int cmin = 1 + (grid - nu) / nu;                      // smallest CTA group
    int r = fit_ring(a, max_tiles(a.gu.nrows, cmin, a.gu.rows_per_tile), max_tiles(a.dn.nrows, cmin, a.dn.rows_per_tile),
                     why);
    if (r) return r;
    a.gu.n_tile_warps = a.n_tile_warps;
    a.dn.n_tile_warps = a.n_tile_warps;
    smem = static_cast<size_t>(a.ctrl_bytes) + a.act_bytes + static_cast<size_t>(a.n_stages) * a.stage_bytes;
    const cudaError_t e = launch_by_type(type, a, grid, smem, st);
    if (e != cudaSuccess) { *cuda_err = e; *why = "stack kernel launch"; return -3; }
    return 0;
}

bool stack_mix_supported(int t) { return stack_mix_slot(t) >= 0; }

int launch_stack_mixed(unsigned used_a, unsigned used_b, StackArgs &a, cudaStream_t st, const char **why,
                       cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    if (a.k > STACK_MAX_K) { *why = "the stack kernel handles k <= 32"; return -2; }
    if (!used_a || !used_b || (used_a | used_b) >> STACK_MIX_TYPES) { *why = "no types for the mixed stack"; return -2; }
    const int H = a.dn.nrows, F = a.gu.nrows;
    int grid = 0;
    uint32_t stage = 0, act = 0, ctrl = 0;
    int n_rb = 0;
    int max_a = 0, max_b = 0;
    const int nu = a.k + (a.has_shared ? 1 : 0);
    // each type in use planned as the layer kernel plans a layer of that type
    for (int s = 0; s < STACK_MIX_TYPES; ++s) {
        const int t = stack_mix_type(s);
        Layer2Args p{};
        p.gu = a.gu;
        p.dn = a.dn;
        p.gu.row_bytes = static_cast<uint32_t>(H / 256 * mix_block_bytes(t));
        p.dn.row_bytes = static_cast<uint32_t>(F / 256 * mix_block_bytes(t));
        p.n_tok = 1;
        p.k = a.k;
        p.n_experts = a.n_experts;
        p.timeout_ns = a.timeout_ns;
        size_t smem = 0;
        const bool in_a = used_a >> s & 1u, in_b = used_b >> s & 1u;
        if (!in_a && !in_b) {
            a.gum[s] = a.dnm[s] = GemvArgs{};
            continue;
        }
        const int rc = plan_layer2(t, t, p, &grid, &smem, why);
        if (rc) return rc;
        // One type's large gate/up tiles would size every stage: Q6_K's
        // smallest whole pass (4 rows of 2,520 bytes, twice) needs 20 KB and
        // leaves 11 stages for all layers. Such a type takes fewer rows per
        // tile (part of a pass idle); its tiles spread over more warps, so
        // the passes per warp stay the same and the ring keeps 16 stages.
        if (2u * p.gu.part_bytes > kMixStageCap) {
            const int rpt = std::max(1, static_cast<int>((kMixStageCap / 2 - 32u) / p.gu.row_bytes));
            if (rpt < p.gu.rows_per_tile) {
                p.gu.rows_per_tile = rpt;
                p.gu.part_bytes =
                    static_cast<uint32_t>((static_cast<uint64_t>(rpt) * p.gu.row_bytes + 15u) & ~15ull) + 32u;
            }
        }
        a.gum[s] = p.gu;
        a.dnm[s] = p.dn;
        const int cmin = 1 + (grid - nu) / nu;
        if (in_a) {
            stage = std::max(stage, 2u * p.gu.part_bytes);
            max_a = std::max(max_a, max_tiles(F, cmin, p.gu.rows_per_tile));
        }
        if (in_b) {
            const uint32_t part_b =
                static_cast<uint32_t>((static_cast<uint64_t>(p.dn.rows_per_tile) * p.dn.row_bytes + 15u) & ~15ull) + 32u;
            stage = std::max(stage, part_b);
            max_b = std::max(max_b, max_tiles(H, cmin, p.dn.rows_per_tile));
        }
        act = std::max(act, p.act_bytes);
        ctrl = std::max(ctrl, p.ctrl_bytes);
        n_rb = p.n_rb;
        a.timeout_ns = p.timeout_ns;
    }
    a.n_rb = n_rb;
    a.stage_bytes = stage;
    a.act_bytes = act;
    a.route_off = ctrl;
    a.ctrl_bytes = (ctrl + static_cast<uint32_t>(sizeof(StackShared)) + 127u) & ~127u;
    int r = fit_ring(a, max_a, max_b, why);
    if (r) return r;
    for (int s = 0; s < STACK_MIX_TYPES; ++s) {
        a.gum[s].n_tile_warps = a.dnm[s].n_tile_warps = a.n_tile_warps;
        a.dnm[s].part_bytes = stage;
    }
    // the first type in use stands in for the shapes and the unit plan
    for (int s = 0; s < STACK_MIX_TYPES; ++s)
        if (used_a >> s & 1u) { a.gu = a.gum[s]; break; }
    for (int s = 0; s < STACK_MIX_TYPES; ++s)
        if (used_b >> s & 1u) { a.dn = a.dnm[s]; break; }
    const size_t smem = static_cast<size_t>(a.ctrl_bytes) + a.act_bytes + static_cast<size_t>(a.n_stages) * a.stage_bytes;
    const cudaError_t e = launch_by_type(T_STACK_MIXED, a, grid, smem, st);
    if (e != cudaSuccess) { *cuda_err = e; *why = "stack kernel launch"; return -3; }
    return 0;
}

}  // namespace moe
