// moe_layer.cu -- planning and dispatch of the fused layer kernel
// (moe_layer.cuh). The tile geometry of each phase follows the GEMV's
// launcher (moe_gemv.cu) so both paths cut rows the same way.
#include <algorithm>

#include "moe_aux.h"
#include "moe_layer_launch.cuh"

namespace moe {

char g_layer_diag[256];

#define MOE_LAYER_PAIRS(X)                                                                          \
    X(T_Q2_K, T_Q2_K) X(T_Q2_K, T_Q3_K) X(T_Q2_K, T_Q4_K) X(T_Q2_K, T_Q6_K)                         \
    X(T_Q3_K, T_Q2_K) X(T_Q3_K, T_Q3_K) X(T_Q3_K, T_Q4_K) X(T_Q3_K, T_Q6_K)                         \
    X(T_Q4_K, T_Q2_K) X(T_Q4_K, T_Q3_K) X(T_Q4_K, T_Q4_K) X(T_Q4_K, T_Q6_K)                         \
    X(T_Q6_K, T_Q2_K) X(T_Q6_K, T_Q3_K) X(T_Q6_K, T_Q4_K) X(T_Q6_K, T_Q6_K)                         \
    X(T_Q4_0, T_Q4_0) X(T_Q5_0, T_Q5_0) X(T_Q8_0, T_Q8_0) X(T_Q5_K, T_Q5_K)

#define MOE_LAYER_DECLARE(A, B)                                                                    \
    extern template cudaError_t launch_layer_t<A, B>(const LayerArgs &, int, size_t, cudaStream_t); \
    extern template cudaError_t launch_layer2_t<A, B>(const Layer2Args &, int, size_t, cudaStream_t);
MOE_LAYER_PAIRS(MOE_LAYER_DECLARE)

namespace {

constexpr int kSmemLimit = 227 * 1024;
constexpr int kTargetStage = 8 * 1024;

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
bool pair_supported(int ta, int tb) {
#define MOE_LAYER_MATCH(A, B) if (ta == A && tb == B) return true;
    MOE_LAYER_PAIRS(MOE_LAYER_MATCH)
#undef MOE_LAYER_MATCH
    return false;
}
int lanes_for(int K, int t) {
    const int T = (K / qk_of(t)) * tasks_of(t);
    int L = 32;
    while (L > 1 && T % L) L >>= 1;
    return L;
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
uint32_t round16(uint64_t x) { return static_cast<uint32_t>((x + 15u) & ~uint64_t{15}); }

}  // namespace

int plan_layer(int ta, int tb, LayerArgs &a, int *grid_out, size_t *smem_out, const char **why) {
    if (!pair_supported(ta, tb)) { *why = "no fused kernel for this gate/up, down type pair"; return -2; }
    const int H = a.gu.K, F = a.gu.nrows, n_tok = a.n_tok, k = a.k;
    const int N = n_tok * k;
    if (n_tok < 1 || n_tok > 8 || k < 1 || k > 32 || N > LAYER_MAX_ENTRIES) {
        *why = "fused layer handles n_tok <= 8, k <= 32, n_tok * k <= 64";
        return -2;
    }
    if (a.dn.K != F || a.dn.nrows != H) { *why = "down shape does not match"; return -2; }
    if (H % qk_of(ta) || F % qk_of(tb)) { *why = "H / F not a multiple of the block size"; return -2; }
    const uint32_t rbA = static_cast<uint32_t>((H / qk_of(ta)) * bytes_of(ta));
    const uint32_t rbB = static_cast<uint32_t>((F / qk_of(tb)) * bytes_of(tb));
    if (a.gu.row_bytes != rbA || a.dn.row_bytes != rbB) { *why = "rows are not contiguous"; return -2; }
    const bool shared = a.gu.shared_up != nullptr;
    const int LA = lanes_for(H, ta), RPA = 32 / LA;
    int LB = lanes_for(F, tb);
    if (LB > 16) LB = 16;                      // phase B runs on half-warps
    const int RPB = 16 / LB;
    const int G = sm_count();

    // phase A tiles: as the GEMV, for the routed groups' upper bound
    const int64_t groups = (N < a.n_experts ? N : a.n_experts) + (shared ? 1 : 0);
    const int64_t rows_cta = (groups * F + G - 1) / G;
    int rpt_max = (kTargetStage / static_cast<int>(2 * rbA)) / RPA * RPA;
    if (rpt_max < RPA) rpt_max = RPA;
    int rpt = static_cast<int>(rows_cta / GEMV_CONSUMER_WARPS) / RPA * RPA;
    if (rpt < RPA) rpt = RPA;
    if (rpt > rpt_max) rpt = rpt_max;
    if (rpt > F) rpt = F;
    const uint32_t part_a = round16(static_cast<uint64_t>(rpt) * rbA) + 32u;
    uint32_t stage = 2 * part_a;
    // phase B tiles: rows of one group within [h0, h1), run by half-warps
    // (RPB rows per pass), two tiles per stage. Aim for ~32 tiles per CTA so
    // every half-warp has one.
    const int hb = (H + G - 1) / G;
    const int ga = static_cast<int>(groups);
    const int tpg_target = (32 + ga - 1) / ga;
    int rows_b = (hb + tpg_target - 1) / tpg_target;
    rows_b = (rows_b + RPB - 1) / RPB * RPB;
    uint32_t part_b = round16(static_cast<uint64_t>(rows_b) * rbB) + 32u;
    if (stage < 2 * part_b) {
        // a smaller phase-B tile fits the stage, or the stage grows
        const int fit = static_cast<int>((stage / 2 - 32u) / rbB) / RPB * RPB;
        if (fit >= RPB) {
            rows_b = fit;
            part_b = round16(static_cast<uint64_t>(rows_b) * rbB) + 32u;
        } else {
            stage = 2 * part_b;
        }
    }
    const uint32_t slot_a = round16(static_cast<uint64_t>(H) + H / 8 + H / 8);
    const uint32_t slot_b = round16(static_cast<uint64_t>(F) + F / 8 + F / 8);
    const uint64_t act_a = static_cast<uint64_t>(n_tok) * slot_a;
    const uint64_t act_b = static_cast<uint64_t>(N + (shared ? n_tok : 0)) * slot_b;
    const uint32_t act = static_cast<uint32_t>(((act_a > act_b ? act_a : act_b) + 127u) & ~uint64_t{127});
    const uint32_t ctrl = (2u * GEMV_MAX_STAGES * 8u + static_cast<uint32_t>(sizeof(LayerCtrl)) + 127u) & ~127u;
    const int64_t avail = kSmemLimit - static_cast<int64_t>(ctrl) - act;
    int S = avail > 0 ? static_cast<int>(avail / stage) : 0;
    if (S > GEMV_MAX_STAGES) S = GEMV_MAX_STAGES;
    if (S < 2) { *why = "activations and tiles do not fit in shared memory"; return -2; }
    const int nw = S >= GEMV_CONSUMER_WARPS ? GEMV_CONSUMER_WARPS : S;   // stage s -> warp s % nw
    S = S / nw * nw;

    a.gu.lanes_per_row = LA;
    a.gu.rows_per_tile = rpt;
    a.gu.n_parts = 2;
    a.gu.n_tile_warps = nw;
    a.gu.part_bytes = part_a;
    a.gu.slot_bytes = slot_a;
    a.dn.lanes_per_row = LB;
    a.dn.rows_per_tile = rows_b;
    a.dn.n_parts = 1;
    a.dn.n_tile_warps = nw;
    a.dn.part_bytes = stage;
    a.dn.slot_bytes = slot_b;
    a.rows_b = rows_b;
    a.part_bytes_b = part_b;
    a.n_stages = S;
    a.stage_bytes = stage;
    a.ctrl_bytes = ctrl;
    a.act_bytes = act;
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;
    *grid_out = G;
    *smem_out = static_cast<size_t>(ctrl) + act + static_cast<size_t>(S) * stage;
    return 0;
}

int launch_layer(int ta, int tb, LayerArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    int grid = 0;
    size_t smem = 0;
    const int rc = plan_layer(ta, tb, a, &grid, &smem, why);
    if (rc) return rc;
    cudaError_t e = cudaErrorInvalidValue;
#define MOE_LAYER_LAUNCH(A, B) else if (ta == A && tb == B) e = launch_layer_t<A, B>(a, grid, smem, st);
    if (false) {}
    MOE_LAYER_PAIRS(MOE_LAYER_LAUNCH)
#undef MOE_LAYER_LAUNCH
    if (e != cudaSuccess) { *cuda_err = e; *why = g_layer_diag; return -3; }
    return 0;
}

// Geometry of the per-expert-group kernel. Every unit gets at least
// floor(G / units) CTAs, so a CTA holds at most ceil(F / that) gate/up rows
// and ceil(H / that) down rows; tiles are sized so those spread over the
// consumer warps, stages hold one gate/up tile (two parts) or one down tile,
// and the tile-warp count nw is chosen so the most stages fit (the stage
// count is a multiple of nw: stage i % S always goes to warp i % nw).
int plan_layer2(int ta, int tb, Layer2Args &a, int *grid_out, size_t *smem_out, const char **why) {
    if (!pair_supported(ta, tb)) { *why = "no fused kernel for this gate/up, down type pair"; return -2; }
    const int H = a.gu.K, F = a.gu.nrows, n_tok = a.n_tok, k = a.k;
    const int N = n_tok * k;
    if (n_tok < 1 || n_tok > 8 || k < 1 || k > 32 || N > LAYER_MAX_ENTRIES) {
        *why = "fused layer handles n_tok <= 8, k <= 32, n_tok * k <= 64";
        return -2;
    }
    if (a.dn.K != F || a.dn.nrows != H) { *why = "down shape does not match"; return -2; }
    if (H % qk_of(ta) || F % qk_of(tb)) { *why = "H / F not a multiple of the block size"; return -2; }
    const uint32_t rbA = static_cast<uint32_t>((H / qk_of(ta)) * bytes_of(ta));
    const uint32_t rbB = static_cast<uint32_t>((F / qk_of(tb)) * bytes_of(tb));
    if (a.gu.row_bytes != rbA || a.dn.row_bytes != rbB) { *why = "rows are not contiguous"; return -2; }
    const bool shared = a.gu.shared_up != nullptr;
    const int G = sm_count();
    const int units = (N < a.n_experts ? N : a.n_experts) + (shared ? 1 : 0);
    if (units > G) { *why = "more experts than SMs"; return -2; }
    const int LA = lanes_for(H, ta), RPA = 32 / LA;
    const int LB = lanes_for(F, tb), RPB = 32 / LB;
    const int ctas = G / units;
    const int rows_a = (F + ctas - 1) / ctas, rows_b_cta = (H + ctas - 1) / ctas;
    int rpt_max = (kTargetStage / static_cast<int>(2 * rbA + 64)) / RPA * RPA;
    if (rpt_max < RPA) rpt_max = RPA;
    int rpt = (rows_a + GEMV_CONSUMER_WARPS - 1) / GEMV_CONSUMER_WARPS;
    rpt = (rpt + RPA - 1) / RPA * RPA;
    if (rpt > rpt_max) rpt = rpt_max;
    if (rpt > F) rpt = F;
    const uint32_t part_a = round16(static_cast<uint64_t>(rpt) * rbA) + 32u;
    uint32_t stage = 2 * part_a;
    int rows_b = (rows_b_cta + GEMV_CONSUMER_WARPS - 1) / GEMV_CONSUMER_WARPS;
    rows_b = (rows_b + RPB - 1) / RPB * RPB;
    while (rows_b > RPB && round16(static_cast<uint64_t>(rows_b) * rbB) + 32u > stage) rows_b -= RPB;
    if (rows_b > H) rows_b = H;
    const uint32_t part_b = round16(static_cast<uint64_t>(rows_b) * rbB) + 32u;
    if (part_b > stage) stage = part_b;
    const uint32_t slot_a = round16(static_cast<uint64_t>(H) + H / 8 + H / 8);
    const uint32_t slot_b = round16(static_cast<uint64_t>(F) + F / 8 + F / 8);
    uint64_t act64 = static_cast<uint64_t>(n_tok) * (slot_a > slot_b ? slot_a : slot_b);
    // expert-parallel: the area first holds every GPU's router logits (f32 [world][E])
    if (a.ep_on) act64 = std::max<uint64_t>(act64, 4ull * n_tok * static_cast<uint64_t>(a.n_experts));
    const uint32_t act = static_cast<uint32_t>((act64 + 127u) & ~uint64_t{127});
    const uint32_t ctrl = (2u * GEMV_MAX_STAGES * 8u + static_cast<uint32_t>(sizeof(Layer2Ctrl)) + 127u) & ~127u;
    const int64_t avail = kSmemLimit - static_cast<int64_t>(ctrl) - act;
    int fit = avail > 0 ? static_cast<int>(avail / stage) : 0;
    if (fit > GEMV_MAX_STAGES) fit = GEMV_MAX_STAGES;
    if (fit < 2) { *why = "activations and tiles do not fit in shared memory"; return -2; }
    int nw = fit < GEMV_CONSUMER_WARPS ? fit : GEMV_CONSUMER_WARPS, S = fit / nw * nw;
    for (int w = nw - 1; w >= 8 && w <= fit; --w)
        if (fit / w * w > S) { S = fit / w * w; nw = w; }

    a.gu.lanes_per_row = LA;
    a.gu.rows_per_tile = rpt;
    a.gu.n_parts = 2;
    a.gu.n_tile_warps = nw;
    a.gu.part_bytes = part_a;
    a.gu.slot_bytes = slot_a;
    a.dn.lanes_per_row = LB;
    a.dn.rows_per_tile = rows_b;
    a.dn.n_parts = 1;
    a.dn.n_tile_warps = nw;
    a.dn.part_bytes = stage;
    a.dn.slot_bytes = slot_b;
    a.n_tile_warps = nw;
    a.n_stages = S;
    a.stage_bytes = stage;
    a.ctrl_bytes = ctrl;
    a.act_bytes = act;
    a.n_rb = (H + LAYER2_RB - 1) / LAYER2_RB;
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;
    *grid_out = G;
    *smem_out = static_cast<size_t>(ctrl) + act + static_cast<size_t>(S) * stage;
    return 0;
}

int launch_layer2(int ta, int tb, Layer2Args &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    int grid = 0;
    size_t smem = 0;
    const int rc = plan_layer2(ta, tb, a, &grid, &smem, why);
    if (rc) return rc;
    cudaError_t e = cudaErrorInvalidValue;
#define MOE_LAYER2_LAUNCH(A, B) else if (ta == A && tb == B) e = launch_layer2_t<A, B>(a, grid, smem, st);
    if (false) {}
    MOE_LAYER_PAIRS(MOE_LAYER2_LAUNCH)
#undef MOE_LAYER2_LAUNCH
    if (e != cudaSuccess) { *cuda_err = e; *why = g_layer_diag; return -3; }
    return 0;
}

}  // namespace moe
