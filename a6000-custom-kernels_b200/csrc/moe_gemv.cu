// moe_gemv.cu -- launch planning and instantiations of the pointer-table GEMV
// (the B200 counterpart of moe_cache_gemv_launch, kernels/moe-cache.cu:781-819).
#include <cstdio>

#include "moe_aux.h"
#include "moe_gemv.cuh"

namespace moe {

namespace {

constexpr int kSmemLimit = 227 * 1024;
constexpr int kActBudget = 96 * 1024;
constexpr int kTargetStage = 8 * 1024;

char g_launch_diag[256];   // attributes of the last failed launch

template <int TYPE, int ACT, int NMX>
cudaError_t launch_t(const GemvArgs &a, int grid, size_t smem, cudaStream_t st) {
    auto kern = moe_gemv_kernel<TYPE, ACT, NMX>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    kern<<<grid, GEMV_THREADS, smem, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        snprintf(g_launch_diag, sizeof(g_launch_diag),
                 "grid=%d threads=%d smem=%zu regs=%d maxThreads=%d maxDynSmem=%d local=%zu", grid, GEMV_THREADS,
                 smem, fa.numRegs, fa.maxThreadsPerBlock, fa.maxDynamicSharedSizeBytes, fa.localSizeBytes);
    }
    return e;
}

template <int TYPE>
cudaError_t dispatch_act(int act, int nmx, const GemvArgs &a, int grid, size_t smem, cudaStream_t st) {
    if (act == ACT_Q8_1) {
        return nmx == 1 ? launch_t<TYPE, ACT_Q8_1, 1>(a, grid, smem, st) : launch_t<TYPE, ACT_Q8_1, 8>(a, grid, smem, st);
    }
    return nmx == 1 ? launch_t<TYPE, ACT_CPU, 1>(a, grid, smem, st) : launch_t<TYPE, ACT_CPU, 8>(a, grid, smem, st);
}

int qk_of(int t) { return is_kquant(t) ? 256 : 32; }
int tasks_of(int t) {
    switch (t) {
        case T_Q2_K: case T_Q3_K: case T_Q6_K: return 2;
        case T_Q4_K: case T_Q5_K: return 4;
        default: return 1;
    }
}
int bytes_of(int t) {
    switch (t) {
        case T_Q4_0: return 18;
        case T_Q5_0: return 22;
        case T_Q8_0: return 34;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

}  // namespace

int launch_gemv(int type, int act, GemvArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    const int qk = qk_of(type), bytes = bytes_of(type);
    if (!bytes) { *why = "unsupported weight type"; return -2; }
    if (a.K <= 0 || a.K % qk) { *why = "ne00 is not a multiple of the block size"; return -1; }
    if (act == ACT_Q8_1 && a.K % 32) { *why = "Q8_1 activations need ne00 % 32 == 0"; return -1; }
    if (a.row_bytes != static_cast<uint32_t>((a.K / qk) * bytes)) { *why = "row stride is not contiguous"; return -2; }
    const int N = a.ncols_dst * a.nchannels_dst;
    if (N <= 0) return 0;
    if (N > GEMV_MAX_ENTRIES) { *why = "ncols_dst * nchannels_dst exceeds 256"; return -2; }
    if (a.ncols_dst > 8) { *why = "ncols_dst exceeds the decode batch limit of 8"; return -2; }
    if (a.nrows <= 0) return 0;

    const int T = (a.K / qk) * tasks_of(type);
    int L = 32;
    while (L > 1 && T % L) L >>= 1;
    const int RP = 32 / L;
    const int parts = a.use_gate ? 2 : 1;
    const bool has_shared_ = a.shared_up != nullptr;
    const int64_t groups_bound_ = (N < a.n_experts ? N : a.n_experts) + (has_shared_ ? 1 : 0);
    const int64_t total_rows = groups_bound_ * a.nrows;
    if (total_rows >= (int64_t{1} << 31)) { *why = "row space of the routed experts exceeds 2^31 rows"; return -2; }
    const int nmx_ = a.ncols_dst == 1 ? 1 : 8;
    if (total_rows * ((N + nmx_ - 1) / nmx_ + 1) >= (int64_t{1} << 32)) { *why = "weighted row space exceeds 2^32"; return -2; }
    const int n_sm_ = sm_count();
    const int64_t grid_ = (total_rows + RP - 1) / RP < n_sm_ ? (total_rows + RP - 1) / RP : n_sm_;
    // tiles small enough that every consumer warp of a CTA gets one, large
    // enough to keep the bulk copies efficient (<= ~8 KB per stage)
    const int64_t rows_cta = (total_rows + grid_ - 1) / grid_;
    int rpt_max = (kTargetStage / static_cast<int>(a.row_bytes * parts)) / RP * RP;
    if (rpt_max < RP) rpt_max = RP;
    int rpt = static_cast<int>(rows_cta / GEMV_CONSUMER_WARPS) / RP * RP;
    if (rpt < RP) rpt = RP;
    if (rpt > rpt_max) rpt = rpt_max;
    if (rpt > a.nrows) rpt = a.nrows;
    const uint32_t part_bytes = ((static_cast<uint32_t>(rpt) * a.row_bytes + 15u) & ~15u) + 32u;
    const uint32_t slot_bytes = (static_cast<uint32_t>(a.K + a.K / 8 + a.K / 8) + 15u) & ~15u;
    const bool has_shared = a.shared_up != nullptr;
    int keys = a.nchannels_y == 1 ? a.ncols_dst : N;
    if (has_shared && a.shared_y) keys += a.ncols_dst;
    int act_cap = kActBudget / static_cast<int>(slot_bytes);
    if (act_cap < a.ncols_dst) act_cap = a.ncols_dst;
    int act_slots = keys < act_cap ? keys : act_cap;
    if (act_slots > GEMV_MAX_KEYS) act_slots = GEMV_MAX_KEYS;
    const uint32_t ctrl = (2u * GEMV_MAX_STAGES * 8u + static_cast<uint32_t>(sizeof(GemvCtrl)) + 127u) & ~127u;
    const int64_t avail = kSmemLimit - static_cast<int64_t>(ctrl) - static_cast<int64_t>(act_slots) * slot_bytes;
    const int64_t stage_bytes = static_cast<int64_t>(part_bytes) * parts;
    int S = avail > 0 ? static_cast<int>(avail / stage_bytes) : 0;
    if (S > GEMV_MAX_STAGES) S = GEMV_MAX_STAGES;
    if (S < 2) { *why = "rows too wide for the shared-memory ring"; return -2; }
    // every stage belongs to one tile warp: S a multiple of the tile warps
    const int nw = S >= GEMV_CONSUMER_WARPS ? GEMV_CONSUMER_WARPS : S;
    S = S / nw * nw;
    const size_t smem = ctrl + static_cast<size_t>(act_slots) * slot_bytes + static_cast<size_t>(S) * stage_bytes;

    a.lanes_per_row = L;
    a.rows_per_tile = rpt;
    a.n_stages = S;
    a.n_tile_warps = nw;
    a.n_parts = parts;
    a.act_slots = act_slots;
    a.part_bytes = part_bytes;
    a.slot_bytes = slot_bytes;
    a.ctrl_bytes = ctrl;
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;

    const int grid = static_cast<int>(grid_);

    const int nmx = a.ncols_dst == 1 ? 1 : 8;
    cudaError_t e;
    switch (type) {
        case T_Q4_0: e = dispatch_act<T_Q4_0>(act, nmx, a, grid, smem, st); break;
        case T_Q5_0: e = dispatch_act<T_Q5_0>(act, nmx, a, grid, smem, st); break;
        case T_Q8_0: e = dispatch_act<T_Q8_0>(act, nmx, a, grid, smem, st); break;
        case T_Q2_K: e = dispatch_act<T_Q2_K>(act, nmx, a, grid, smem, st); break;
        case T_Q3_K: e = dispatch_act<T_Q3_K>(act, nmx, a, grid, smem, st); break;
        case T_Q4_K: e = dispatch_act<T_Q4_K>(act, nmx, a, grid, smem, st); break;
        case T_Q5_K: e = dispatch_act<T_Q5_K>(act, nmx, a, grid, smem, st); break;
        case T_Q6_K: e = dispatch_act<T_Q6_K>(act, nmx, a, grid, smem, st); break;
        default: *why = "unsupported weight type"; return -2;
    }
    if (e != cudaSuccess) { *cuda_err = e; *why = g_launch_diag; return -3; }
    return 0;
}

}  // namespace moe
