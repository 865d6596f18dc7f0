// moe_layer2.cuh -- one MoE layer of decode tokens in ONE launch, split into
// per-expert CTA groups.
//
// The layer is routed experts + the shared expert, each a "unit" (a distinct
// expert with the tokens that picked it). The grid (one CTA per SM,
// cooperative launch) is cut into contiguous CTA groups, one per unit, sized
// by the unit's member count. CTA j of a group of C owns
//   gate/up rows [F j / C, F (j + 1) / C) and down rows [H j / C, H (j + 1) / C)
// of its unit's expert, for every member token. Its producer warp streams all
// of those weights into a shared-memory ring at once -- a batch-1 CTA's
// ~145 KB fit, so every weight byte of the layer is requested within a few
// microseconds of launch -- and the shared expert's CTAs start before routing
// is known, since their weights do not depend on it.
//
// Data exchange stays inside a group: gate/up results h go out as (value,
// launch tag) pairs, and each CTA of the group takes its unit's h (768
// values a member at config 2) as soon as every tag is this launch's. Down
// results y are combined without any wait: output rows are cut into blocks of
// RB rows with one arrival counter per (token, block); a CTA adds the rows it
// wrote, and the CTA whose addition completes a block (k + 1 contributions of
// every row) sums that block in pick order plus the shared expert and resets
// the counter. The per-row arithmetic is the GEMV's (consume_tile), and the
// combine adds in the same order as the combine kernel, so results equal the
// four-launch path bit for bit.
#pragma once
#include "moe_layer.cuh"

namespace moe {

constexpr int LAYER2_RB = 64;            // output rows per combine block

// Optional timeline (built with -DMOE_LAYER2_TRACE): per CTA and mark, the
// global timer (ns) and the SM clock; off by default.
#ifdef MOE_LAYER2_TRACE
__device__ unsigned long long g_layer2_trace[148 * 64];
#define L2_MARK(i)                                                                               \
    do {                                                                                         \
        if (lane == 0) {                                                                         \
            g_layer2_trace[blockIdx.x * 64 + (i)] = global_timer_ns();                           \
            g_layer2_trace[blockIdx.x * 64 + 32 + (i)] = clock64();                              \
        }                                                                                        \
    } while (0)
#else
#define L2_MARK(i) do {} while (0)
#endif
constexpr int LAYER2_ROUTE_WARPS = 4;    // warps routing the single token of a batch-1 launch

// Expert-parallel decode: each GPU owns one buffer, mapped into the others
// (CUDA IPC). Every value crosses as one 64-bit word (float bits | tag << 32,
// tag = exchange epoch + 1), so a reader that sees the tag sees the value:
// no fence, flag or counter. Parts (byte offsets, 256-aligned): gx u64
// [2][W][H] and glog u64 [2][W][E] -- every GPU's token x and router logits,
// written by their owners into slot [parity][src] (parity = epoch & 1);
// yhome u64 [k + 1][H] -- the down rows of this GPU's token, row p < k
// written by the GPU owning pick p's expert, row k the shared expert's;
// epoch u32 -- layer calls through the exchange.
struct EpDecodeLayout {
    uint64_t gx, glog, yhome, epoch, bytes;
};
__host__ __device__ inline EpDecodeLayout ep_decode_layout(int H, int E, int k, int W) {
    auto up = [](uint64_t x) { return (x + 255u) & ~uint64_t{255}; };
    EpDecodeLayout L;
    uint64_t off = 0;
    L.gx = off;     off += up(8ull * 2 * W * H);
    L.glog = off;   off += up(8ull * 2 * W * E);
    L.yhome = off;  off += up(8ull * (k + 1) * H);
    L.epoch = off;  off += 256;
    L.bytes = off;
    return L;
}

__device__ __forceinline__ uint64_t tagged(float v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64x2(uint64_t *p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_relaxed_sys_u64x2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// One activation block of tagged words (a Q8_K block of 256 or a Q8_0 block
// of 32) in the lane layout of load_q8K_vals / stage_q80_block; true when
// every word of the lane carries `tag`.
template <bool KQ>
__device__ __forceinline__ bool load_tagged_block(const uint64_t *xb, uint32_t tag, int lane,
                                                  float (&v)[KQ ? 8 : 1]) {
    constexpr int NV = KQ ? 8 : 1;
    uint64_t w[NV];
    if constexpr (KQ) {
        ld_relaxed_sys_u64x2(xb + 4 * lane, w[0], w[1]);
        ld_relaxed_sys_u64x2(xb + 4 * lane + 2, w[2], w[3]);
        ld_relaxed_sys_u64x2(xb + 128 + 4 * lane, w[4], w[5]);
        ld_relaxed_sys_u64x2(xb + 128 + 4 * lane + 2, w[6], w[7]);
    } else {
        uint64_t other;
        ld_relaxed_sys_u64x2(xb + (lane & ~1), w[0], other);
        if (lane & 1) w[0] = other;
    }
    bool ok = true;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        ok &= static_cast<uint32_t>(w[j] >> 32) == tag;
        v[j] = __uint_as_float(static_cast<uint32_t>(w[j]));
    }
    return ok;
}
constexpr int EP_DECODE_MAX_WORLD = 8;
struct EpDecodeArgs {
    int32_t world, rank;                 // one token per GPU: token t lives on GPU t
    int32_t expert_lo, n_local;          // this GPU's experts [expert_lo, expert_lo + n_local)
    char *peer[EP_DECODE_MAX_WORLD];     // every GPU's exchange buffer as seen from this GPU
    EpDecodeLayout lay;
};

struct Layer2Args {
    GemvArgs gu, dn;                     // per-phase shapes, tile geometry, outputs
    LayerTensor up, gate, down;
    const char *shared_down;
    int32_t tma_shared_down;
    const float *logits;
    int32_t n_tok, k, n_experts, norm_w;
    int32_t *ids_out;
    float *w_out, *out;
    uint32_t *stats;
    const uint32_t *clock;
    uint32_t log_cap;
    uint64_t *h_tag, *hs_tag;            // h / hs as (value, tag) pairs
    uint32_t *gbar;                      // [0] launch epoch, [1] finished CTAs
    uint32_t *rowcnt;                    // [n_tok][n_rb] rows arrived per combine block (zero between launches)
    int32_t n_rb;
    int32_t n_stages, n_tile_warps;
    uint32_t stage_bytes, ctrl_bytes, act_bytes;
    int *err;
    uint64_t timeout_ns;
    int32_t ep_on;                       // expert-parallel decode (ep below); n_tok = world
    uint64_t ep_timeout_ns;              // limit of the waits for other GPUs
    EpDecodeArgs ep;
};

struct Layer2Ctrl {
    GemvCtrl g;
    const char *dsrc[LAYER_MAX_ENTRIES];
    uint8_t dkind[LAYER_MAX_ENTRIES], dhost[LAYER_MAX_ENTRIES];
    float wt[LAYER_MAX_ENTRIES];
    uint32_t cand_key[512];
    int32_t cand_id[512];
    uint32_t uw[LAYER_MAX_ENTRIES + 2];  // prefix of unit weights (members)
    int32_t gid[LAYER_MAX_ENTRIES];      // routed experts (global ids; C.x holds local ones)
    uint32_t tag, xep;                   // launch tag; expert-parallel exchange epoch
    uint32_t halt;                       // persistent stack kernel: stop at this layer (a wait ran out)
};

// This CTA's place in the unit partition. Unit u (of nu) gets CTAs
// [c_u, c_{u+1}) with c_u = u + floor((G - nu) * W_u / W), W_u the prefix of
// the unit weights (pre == nullptr: every unit weighs 1), so every unit has
// at least one CTA and the rest are shared by weight.
struct UnitPlan {
    int u, j, c;                         // unit, index in its group, group size
    int a0, a1, b0, b1;                  // gate/up rows, down rows
    int nA, nB;                          // tiles of each phase
};

__device__ __forceinline__ int unit_first_cta(int u, int nu, int G, const uint32_t *pre) {
    const uint64_t Wu = pre ? pre[u] : static_cast<uint64_t>(u);
    const uint64_t W = pre ? pre[nu] : static_cast<uint64_t>(nu);
    return u + static_cast<int>((static_cast<uint64_t>(G - nu) * Wu) / W);
}

__device__ __forceinline__ UnitPlan unit_plan(int nu, const uint32_t *pre, int G, int bid, int F, int H, int rpt,
                                              int rows_b) {
    UnitPlan P;
    int lo = 0, hi = nu - 1;             // last u with c_u <= bid
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (unit_first_cta(mid, nu, G, pre) <= bid) lo = mid;
        else hi = mid - 1;
    }
    P.u = lo;
    const int c0 = unit_first_cta(lo, nu, G, pre);
    const int c1 = lo + 1 < nu ? unit_first_cta(lo + 1, nu, G, pre) : G;
    P.j = bid - c0;
    P.c = c1 - c0;
    P.a0 = static_cast<int>(static_cast<int64_t>(F) * P.j / P.c);
    P.a1 = static_cast<int>(static_cast<int64_t>(F) * (P.j + 1) / P.c);
    P.b0 = static_cast<int>(static_cast<int64_t>(H) * P.j / P.c);
    P.b1 = static_cast<int>(static_cast<int64_t>(H) * (P.j + 1) / P.c);
    P.nA = (P.a1 - P.a0 + rpt - 1) / rpt;
    P.nB = (P.b1 - P.b0 + rows_b - 1) / rows_b;
    return P;
}

// Selection of NV-wide slices (NV = experts per lane in a warp's slice).
template <int NV>
__device__ __forceinline__ void route_slices_nv(const float *l, int n_experts, int k, int w, int lane,
                                                uint32_t *ck, int *ci) {
    route_block_slices<NV>(l, n_experts, k, w, lane, ck, ci);
}
__device__ __forceinline__ bool route_slices(const float *l, int n_experts, int k, int w, int nw, int lane,
                                             uint32_t *ck, int *ci) {
    const int per = (n_experts + 32 * nw - 1) / (32 * nw);
    if (per <= 1) route_slices_nv<1>(l, n_experts, k, w, lane, ck, ci);
    else if (per <= 2) route_slices_nv<2>(l, n_experts, k, w, lane, ck, ci);
    else if (per <= 4) route_slices_nv<4>(l, n_experts, k, w, lane, ck, ci);
    else if (per <= 8) route_slices_nv<8>(l, n_experts, k, w, lane, ck, ci);
    else if (per <= 16) route_slices_nv<16>(l, n_experts, k, w, lane, ck, ci);
    else return false;
    return true;
}


template <int TA, int TB>
__global__ void __launch_bounds__(GEMV_THREADS, 1) moe_layer2_kernel(const __grid_constant__ Layer2Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    Layer2Ctrl &LC = *reinterpret_cast<Layer2Ctrl *>(smem + 2 * GEMV_MAX_STAGES * 8);
    GemvCtrl &C = LC.g;
    uint8_t *act_area = smem + a.ctrl_bytes;
    uint8_t *stage_area = act_area + a.act_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.n_stages, k = a.k, n_tok = a.n_tok, N = n_tok * k, E = a.n_experts;
    const int H = a.dn.nrows, F = a.gu.nrows, KA = a.gu.K, KB = a.dn.K;
    const bool has_shared = a.gu.shared_up != nullptr;
    const int hs = has_shared ? 1 : 0;
    const int G = gridDim.x, bid = blockIdx.x;
    const int rpt = a.gu.rows_per_tile, rows_b = a.dn.rows_per_tile;
    constexpr int PW = GEMV_CONSUMER_WARPS;          // the producer warp
    const bool epm = a.ep_on != 0;                   // expert-parallel decode (n_tok = world)
    const int me = epm ? a.ep.rank : 0;
    const int lo_e = epm ? a.ep.expert_lo : 0, n_loc = epm ? a.ep.n_local : E;
    const int n_sh = epm ? 1 : n_tok;                // tokens of the shared expert (this GPU's own in EP)
    const bool one = n_tok == 1 && !epm;
    // the routed tokens' x and logits: the caller's, or (EP) every GPU's
    // token from this GPU's gather slots
    const float *x_base = reinterpret_cast<const float *>(a.gu.y);
    const float *lg_base = a.logits;
    const uint64_t *x_tag = nullptr;                 // EP: every GPU's token x as tagged words
    uint32_t ep_tag = 0;
    if (warp == 0) L2_MARK(0);
    if (warp == PW) L2_MARK(13);

    auto src_of = [&](const LayerTensor &T, int x, const char *&src, uint8_t &kind, uint8_t &host) {
        if (T.tbl) {
            const uintptr_t p = reinterpret_cast<uintptr_t>(T.tbl[x]);
            src = reinterpret_cast<const char *>(p & ~static_cast<uintptr_t>(1));
            host = static_cast<uint8_t>(p & 1u);
        } else {
            src = T.dense + static_cast<uint64_t>(x) * T.expert_bytes;
            host = 0;
        }
        kind = static_cast<uint8_t>(host ? (T.tma ? 1 : 2) : (T.tma ? 0 : 2));
    };
    auto resolve = [&](int u, int x) {
        src_of(a.up, x, C.usrc[u][0], C.ukind[u][0], C.uhost[u][0]);
        src_of(a.gate, x, C.usrc[u][1], C.ukind[u][1], C.uhost[u][1]);
        src_of(a.down, x, LC.dsrc[u], LC.dkind[u], LC.dhost[u]);
    };
    // the producer's description of tile i of unit plan P (phase A, then B)
    auto describe = [&](const UnitPlan &P, int i, TileSrc &ts) {
        const int U = C.n_unique;
        const bool routed = P.u < U;
        if (i < P.nA) {
            ts.row0[0] = ts.row0[1] = P.a0 + i * rpt;
            ts.nr[0] = ts.nr[1] = min(rpt, P.a1 - ts.row0[0]);
            ts.src[0] = routed ? C.usrc[P.u][0] : a.gu.shared_up;
            ts.src[1] = routed ? C.usrc[P.u][1] : a.gu.shared_gate;
            ts.kind[0] = routed ? C.ukind[P.u][0] : (a.gu.tma_shared ? 0 : 2);
            ts.kind[1] = routed ? C.ukind[P.u][1] : (a.gu.tma_shared ? 0 : 2);
            ts.n_parts = 2;
            ts.rb = a.gu.row_bytes;
            ts.part_bytes = a.gu.part_bytes;
        } else {
            const int j = i - P.nA;
            ts.row0[0] = ts.row0[1] = P.b0 + j * rows_b;
            ts.nr[0] = ts.nr[1] = min(rows_b, P.b1 - ts.row0[0]);
            ts.src[0] = ts.src[1] = routed ? LC.dsrc[P.u] : a.shared_down;
            ts.kind[0] = ts.kind[1] = routed ? LC.dkind[P.u] : (a.tma_shared_down ? 0 : 2);
            ts.n_parts = 1;
            ts.rb = a.dn.row_bytes;
            ts.part_bytes = a.stage_bytes;
        }
    };
    auto produce = [&](const UnitPlan &P) {
        produce_tiles(P.nA + P.nB, S, full, empty, stage_area, a.stage_bytes,
                      [&](int i, TileSrc &ts) { describe(P, i, ts); }, a.timeout_ns, a.err, lane);
    };
    // x of token t into activation slot t (llama.cpp CPU quantization)
    auto stage_x = [&](int t, int b) {
        uint8_t *slot = act_area + static_cast<size_t>(t) * a.gu.slot_bytes;
        if (!x_tag) {
            stage_f32_block<TA>(x_base + static_cast<int64_t>(t) * a.gu.stride_col_y, slot, KA, b, lane);
            return;
        }
        // EP: the gathered token, polled until every word carries this call's tag
        constexpr bool KQ = is_kquant(TA);
        constexpr int QB = KQ ? 256 : 32;
        const uint64_t *xb = x_tag + static_cast<int64_t>(t) * KA + b * QB;
        float v[KQ ? 8 : 1];
        const uint64_t t0 = clock64(), lim = timeout_cycles(a.ep_timeout_ns);
        while (!__all_sync(0xffffffffu, load_tagged_block<KQ>(xb, ep_tag, lane, v))) {
            if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
                break;
            }
        }
        int8_t *q = reinterpret_cast<int8_t *>(slot);
        int16_t *bs = reinterpret_cast<int16_t *>(slot + KA);
        float *sc = reinterpret_cast<float *>(slot + KA + KA / 8);
        if constexpr (KQ) quant_q8K_vals<TA>(v, q, bs, sc, b, lane, KA / chunk_of<TA>::CE);
        else quant_q80_val<TA>(v[0], q, bs, sc, b, lane, KA / chunk_of<TA>::CE);
    };
    constexpr int QA = is_kquant(TA) ? 256 : 32;
    const int nbx = KA / QA;

    // ---- 1. routing, units, plan --------------------------------------------
    UnitPlan P{};
    bool early = false;                   // a batch-1 CTA of the shared expert
    uint32_t tokmask = 0;                 // tokens whose x (and weights) this CTA needs
    if (one) {
        // One token: its k picks are distinct, so unit u = pick u and the
        // shared expert is unit k whatever the routing: the plan is fixed
        // before the logits are read, and the shared expert's CTAs stream at once.
        P = unit_plan(k + hs, nullptr, G, bid, F, H, rpt, rows_b);
        tokmask = 1u;
        early = has_shared && P.u == k;
        if (warp == PW) {
            for (int s = lane; s < S; s += 32) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            fence_mbar_init();
            __syncwarp();
            // the consumers wait on named barrier 3 for the initialised ring
            asm volatile("bar.arrive 3, %0;" ::"r"(GEMV_THREADS) : "memory");
            if (early) {
                C.n_unique = k;           // read by describe(); thread 0 writes the same value
                produce(P);
            } else {
                asm volatile("bar.sync 4, 64;" ::: "memory");   // the routing warp's picks and sources
                L2_MARK(5);
                if (!C.fail) produce(P);
            }
            return;
        }
        // Routed CTAs: every consumer warp takes a slice of the logits, warp
        // PW - 1 merges, records the groups and hands the sources to the
        // producer (named barrier 4) while the others quantize x. The
        // shared expert's CTAs quantize x and start on their tiles at once;
        // they route later (their routing only feeds the gating weights).
        if (!early) {
            // E <= 512, k <= 8: rank selection (no serial rounds); else slices + merge
            const bool ranked = E <= 32 * PW && k <= 8;
            bool sliced = false;
            if (ranked) rank_slice(a.logits, E, k, warp, lane, LC.cand_key, LC.cand_id);
            else sliced = k <= 16 && route_slices(a.logits, E, k, warp, PW, lane, LC.cand_key, LC.cand_id);
            if (warp == PW - 1) L2_MARK(1);
            consumer_sync();
            if (ranked) {
                rank_candidates(LC.cand_key, LC.cand_id, PW * k, k, tid, C.x);
                consumer_sync();
            }
            if (warp == PW - 1) {
                L2_MARK(2);
                if (!ranked) {
                    if (sliced) merge_topk(LC.cand_key, LC.cand_id, PW * k, k, lane, C.x);
                    else route_select(a.logits, E, k, lane, C.x);
                    __syncwarp();
                }
                L2_MARK(3);
                bool bad = false;
                if (lane < k) {
                    const int x = C.x[lane];
                    bad = x < 0 || x >= E;
                    C.first[lane] = static_cast<int16_t>(lane);
                    C.uidx[lane] = static_cast<int16_t>(lane);
                    C.gmem[lane] = static_cast<int16_t>(lane);
                    C.goff[lane] = static_cast<int16_t>(lane);
                    C.uexp[lane] = x;
                    C.eslot[lane] = 0;
                    if (!bad) resolve(lane, x);
                }
                if (lane < k) LC.gid[lane] = C.x[lane];
                bad = __any_sync(0xffffffffu, bad);
                if (lane == 0) {
                    C.n_unique = k;
                    C.goff[k] = static_cast<int16_t>(k);
                    C.shslot[0] = 0;
                    C.fail = bad ? 1 : 0;
                    if (bad) set_error(a.err, DERR_BAD_ID);
                }
                __syncwarp();
                L2_MARK(4);
                asm volatile("bar.arrive 4, 64;" ::: "memory");
            }
        } else if (tid == 0) {
            C.fail = 0;
            C.n_unique = k;               // the producer wrote the same value for itself
            C.goff[k] = static_cast<int16_t>(k);
            C.shslot[0] = 0;
        }
        if (warp < PW - 1)
            for (int b = warp; b < nbx; b += PW - 1) stage_x(0, b);
        if (warp == 0) L2_MARK(6);
        if (tid == 0) LC.tag = ld_relaxed_u32(&a.gbar[0]) + 1u;
        asm volatile("bar.sync 3, %0;" ::"r"(GEMV_THREADS) : "memory");   // consumers + the producer's arrival
        if (warp == 0) L2_MARK(7);
    } else {
        // Several tokens: GW warps route each token over slices, one merges;
        // the picks are grouped by expert (block barriers, the producer
        // included), and the groups weighted by their member counts.
        if (warp == PW) {
            for (int s = lane; s < S; s += 32) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            fence_mbar_init();
        }
        if (tid == 0) {
            C.fail = 0;
            LC.tag = ld_relaxed_u32(&a.gbar[0]) + 1u;
            if (epm) LC.xep = ld_relaxed_u32(reinterpret_cast<const uint32_t *>(a.ep.peer[me] + a.ep.lay.epoch));
        }
        if (epm) {
            // dispatch: CTA d < world writes this GPU's x and logits as
            // tagged words into GPU d's gather slot [parity][me]; then every
            // CTA takes all GPUs' logits from its own slots (polling the
            // tags) into shared memory for routing
            __syncthreads();
            const uint32_t xep = LC.xep, etag = xep + 1u;
            const int W = n_tok, par = static_cast<int>(xep & 1u);
            const EpDecodeLayout &Ly = a.ep.lay;
            if (bid < W) {
                char *dst = a.ep.peer[bid];
                uint64_t *gx = reinterpret_cast<uint64_t *>(dst + Ly.gx) + static_cast<int64_t>(par * W + me) * H;
                uint64_t *gl = reinterpret_cast<uint64_t *>(dst + Ly.glog) + static_cast<int64_t>(par * W + me) * E;
                const float2 *x2 = reinterpret_cast<const float2 *>(a.gu.y);
                for (int i = tid; i < H / 2; i += GEMV_THREADS) {
                    const float2 v = x2[i];
                    st_relaxed_sys_u64x2(gx + 2 * i, tagged(v.x, etag), tagged(v.y, etag));
                }
                for (int i = tid; i < E; i += GEMV_THREADS) st_relaxed_sys_u64(gl + i, tagged(a.logits[i], etag));
            }
            if (warp == 0) L2_MARK(15);
            const uint64_t *gl_own = reinterpret_cast<const uint64_t *>(a.ep.peer[me] + Ly.glog) +
                                     static_cast<int64_t>(par) * W * E;
            float *lg_s = reinterpret_cast<float *>(act_area);     // free until x is staged
            const uint64_t t0 = clock64(), lim = timeout_cycles(a.ep_timeout_ns);
            bool late = false;
            for (int i = tid; i < W * E; i += GEMV_THREADS) {
                uint64_t w = ld_relaxed_sys_u64(gl_own + i);
                while (static_cast<uint32_t>(w >> 32) != etag) {
                    if (static_cast<uint64_t>(clock64()) - t0 > lim) { late = true; break; }
                    w = ld_relaxed_sys_u64(gl_own + i);
                }
                lg_s[i] = __uint_as_float(static_cast<uint32_t>(w));
                if (late) break;
            }
            if (late) {
                set_error(a.err, DERR_TIMEOUT_FULL);
                C.fail = 1;
            }
            if (warp == 0) L2_MARK(16);
            x_tag = reinterpret_cast<const uint64_t *>(a.ep.peer[me] + Ly.gx) + static_cast<int64_t>(par) * W * H;
            ep_tag = etag;
            lg_base = lg_s;
        }
        __syncthreads();
        const int GW = PW / n_tok;
        const int per = (E + 32 * GW - 1) / (32 * GW);
        const bool sliced = k <= 16 && per <= 16 && GW * k <= 512;
        if (sliced && warp < GW * n_tok) {
            const int t = warp / GW, w = warp % GW;
            route_slices(lg_base + static_cast<int64_t>(t) * E, E, k, w, GW, lane, LC.cand_key + t * GW * k,
                         LC.cand_id + t * GW * k);
        }
        __syncthreads();
        if (warp < n_tok) {
            const int t = warp;
            if (sliced) merge_topk(LC.cand_key + t * GW * k, LC.cand_id + t * GW * k, GW * k, k, lane, &C.x[t * k]);
            else route_select(lg_base + static_cast<int64_t>(t) * E, E, k, lane, &C.x[t * k]);
        }
        __syncthreads();
        if (warp == 0) L2_MARK(17);
        if (tid < N) LC.gid[tid] = C.x[tid];
        // groups of this GPU's experts (EP: other GPUs' picks leave the grouping)
        build_groups(C, N, n_loc, [&](int e) { return C.x[e] - lo_e; }, resolve, a.err, epm);   // ends with a barrier
        if (warp == 0 && !C.fail) {
            const int U = C.n_unique;
            uint32_t run = 0;
            for (int u0 = 0; u0 <= U + hs; u0 += 32) {
                const int u = u0 + lane;
                uint32_t w = 0;
                if (u < U) w = static_cast<uint32_t>(C.goff[u + 1] - C.goff[u]);
                else if (u == U && hs) w = static_cast<uint32_t>(n_sh);
                uint32_t incl = w;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += o;
                }
                if (u <= U + hs) LC.uw[u] = run + incl - w;
                run += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        __syncthreads();
        if (!C.fail) {
            P = unit_plan(C.n_unique + hs, LC.uw, G, bid, F, H, rpt, rows_b);
            if (P.u < C.n_unique) {
                for (int m = C.goff[P.u]; m < C.goff[P.u + 1]; ++m) tokmask |= 1u << (C.gmem[m] / k);
            } else {
                tokmask = epm ? 1u << me : (1u << n_tok) - 1u;
            }
        }
        if (warp == 0) L2_MARK(18);
        if (warp == PW) {
            if (!C.fail) produce(P);
            return;
        }
        for (int job = warp; job < n_tok * nbx; job += PW) {
            const int t = job / nbx;
            if ((tokmask >> t) & 1u) stage_x(t, job % nbx);
        }
        for (int e = tid; e < N; e += PW * 32) C.eslot[e] = static_cast<int16_t>(e / k);
        if (tid < n_sh) C.shslot[tid] = static_cast<int16_t>(epm ? me : tid);
        consumer_sync();
    }

    // ============================ consumer warps =============================
    const int U = C.n_unique;
    const bool run = !C.fail;
    const int u = P.u;
    const bool routed = u < U;
    const int nA = run ? P.nA : 0, nB = run ? P.nB : 0;
    const uint32_t tag = LC.tag;
    const int nw = a.n_tile_warps;

    // ---- gating weights of this CTA's tokens (warps from the top) and the
    //      reference kernel's bookkeeping (:163-198, the first CTA) -----------
    // (the first CTA does every token: it publishes the weights)
    // (EP: only this GPU's own token is summed here; its logits are the caller's)
    const uint32_t wmask = epm ? (1u << me) : (bid == 0 ? (1u << n_tok) - 1u : tokmask);
    if (one && early && warp == PW - 1) {
        // the shared expert's CTAs route now, off their critical path
        route_select(a.logits, E, k, lane, LC.gid);
        __syncwarp();
    }
    if (run && warp >= PW - n_tok && ((wmask >> (PW - 1 - warp)) & 1u)) {
        const int t = PW - 1 - warp;
        const float *lw = epm ? a.logits : lg_base + static_cast<int64_t>(t) * E;
        route_weights(lw, E, k, a.norm_w, lane, &LC.gid[t * k], &LC.wt[t * k]);
        __syncwarp();
        if (bid == 0 && lane < k && (!epm || t == me)) a.w_out[(epm ? 0 : t) * k + lane] = LC.wt[t * k + lane];
    }
    if (bid == 0 && run && warp == PW - 1 - n_tok) {
        const uint32_t clk = a.clock ? *a.clock : 0u;
        for (int e = lane; e < N; e += 32) {
            const int x = C.x[e], g = C.uidx[e];
            if (!epm || e / k == me) a.ids_out[epm ? e % k : e] = LC.gid[e];
            if (x < 0) continue;              // another GPU's expert
            const LayerTensor *T[3] = {&a.up, &a.gate, &a.down};
            const uint8_t host[3] = {C.uhost[g][0], C.uhost[g][1], LC.dhost[g]};
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                if (!T[j]->stamps) continue;
                T[j]->stamps[x] = clk;
                if (!a.stats) continue;
                if (host[j]) {
                    const uint32_t s = atomicAdd(a.stats, 1u);
                    if (s < a.log_cap) a.stats[GEMV_LOG_BASE + s] = (static_cast<uint32_t>(T[j]->cache_id) << 12) | x;
                } else {
                    atomicAdd(a.stats + 1, 1u);
                }
            }
        }
    }
    if (bid == 0 && !run && tid == 0) {
        // keep the routing visible even when a bad id stopped the launch
        for (int e = 0; e < N; ++e)
            if (!epm || e / k == me) a.ids_out[epm ? e % k : e] = LC.gid[e];
    }

    // ---- 2a. gate/up + GLU of this CTA's rows -> h (and tagged copies) ------
    for (int i = warp; i < nA && warp < nw; i += nw) {
        const int s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        if (i == 0) L2_MARK(8);
        const int row0 = P.a0 + i * rpt, nr = min(rpt, P.a1 - row0);
        const char *s0 = routed ? C.usrc[u][0] : a.gu.shared_up;
        const char *s1 = routed ? C.usrc[u][1] : a.gu.shared_gate;
        const uint8_t *stage = stage_area + static_cast<size_t>(s) * a.stage_bytes;
        const uint64_t off = static_cast<uint64_t>(row0) * a.gu.row_bytes;
        const uint8_t *up_rows = stage + ((reinterpret_cast<uintptr_t>(s0) + off) & 15u);
        const uint8_t *gate_rows = stage + a.gu.part_bytes + ((reinterpret_cast<uintptr_t>(s1) + off) & 15u);
        consume_tile<TA, ACT_CPU, 1, 2>(a.gu, C, up_rows, gate_rows, nr, u, U, row0, act_area, lane, a.h_tag,
                                        a.hs_tag, tag);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    consumer_sync();
    if (warp == 0) L2_MARK(9);
    // phase-B activation slots: member m of the unit -> slot m
    const int nm = run ? (routed ? C.goff[u + 1] - C.goff[u] : n_sh) : 0;
    if (routed) {
        for (int m = tid; m < nm; m += PW * 32) C.eslot[C.gmem[C.goff[u] + m]] = static_cast<int16_t>(m);
    } else if (tid < n_sh) {
        C.shslot[tid] = static_cast<int16_t>(tid);
    }
    consumer_sync();

    // ---- 2b. the unit's h from the CTAs of its group, quantized for down. A
    //      block is taken once all its values carry this launch's tag; each
    //      warp loads up to 4 blocks before quantizing any ------------------
    {
        constexpr bool KQ = is_kquant(TB);
        constexpr int QB = KQ ? 256 : 32, NV = KQ ? 8 : 1, BATCH = 4;
        const int nb = KB / QB;
        const int njobs = nm * nb;
        auto block_of = [&](int job) -> const uint64_t * {
            const int m = job / nb, b = job % nb;
            const uint64_t *base;
            if (routed) {
                const int e = C.gmem[C.goff[u] + m], t = e / k, p = e % k;
                base = a.h_tag + static_cast<int64_t>(p) * a.dn.stride_channel_y + static_cast<int64_t>(t) * a.dn.stride_col_y;
            } else {
                base = a.hs_tag + static_cast<int64_t>(m) * a.dn.shared_y_stride_col;
            }
            return base + b * QB;
        };
        auto load = [&](const uint64_t *xb, float (&v)[NV]) -> bool {
            uint64_t w[NV];
            if constexpr (KQ) {
                ld_relaxed_u64x2(xb + 4 * lane, w[0], w[1]);
                ld_relaxed_u64x2(xb + 4 * lane + 2, w[2], w[3]);
                ld_relaxed_u64x2(xb + 128 + 4 * lane, w[4], w[5]);
                ld_relaxed_u64x2(xb + 128 + 4 * lane + 2, w[6], w[7]);
            } else {
                uint64_t other;
                ld_relaxed_u64x2(xb + (lane & ~1), w[0], other);
                if (lane & 1) w[0] = other;
            }
            bool ok = true;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                ok &= static_cast<uint32_t>(w[j] >> 32) == tag;
                v[j] = __uint_as_float(static_cast<uint32_t>(w[j]));
            }
            return ok;
        };
        const uint64_t t0 = clock64(), lim = timeout_cycles(a.timeout_ns);
        for (int base = warp; base < njobs; base += PW * BATCH) {
            float vals[BATCH][NV];
            bool ok[BATCH];
#pragma unroll
            for (int r = 0; r < BATCH; ++r) {
                const int job = base + r * PW;
                ok[r] = true;
                if (job < njobs) ok[r] = load(block_of(job), vals[r]);
            }
            for (;;) {
                unsigned waiting = 0;
#pragma unroll
                for (int r = 0; r < BATCH; ++r) {
                    const int job = base + r * PW;
                    if (job < njobs && !__all_sync(0xffffffffu, ok[r])) waiting |= 1u << r;
                }
                if (!waiting) break;
                if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                    if (lane == 0) set_error(a.err, DERR_TIMEOUT_TAG);
                    break;
                }
#pragma unroll
                for (int r = 0; r < BATCH; ++r)
                    if ((waiting >> r) & 1u) ok[r] = load(block_of(base + r * PW), vals[r]);
            }
#pragma unroll
            for (int r = 0; r < BATCH; ++r) {
                const int job = base + r * PW;
                if (job >= njobs) break;
                uint8_t *slot = act_area + static_cast<size_t>(job / nb) * a.dn.slot_bytes;
                int8_t *q = reinterpret_cast<int8_t *>(slot);
                int16_t *bs = reinterpret_cast<int16_t *>(slot + KB);
                float *sc = reinterpret_cast<float *>(slot + KB + KB / 8);
                if constexpr (KQ) quant_q8K_vals<TB>(vals[r], q, bs, sc, job % nb, lane, KB / chunk_of<TB>::CE);
                else quant_q80_val<TB>(vals[r][0], q, bs, sc, job % nb, lane, KB / chunk_of<TB>::CE);
            }
        }
    }
    consumer_sync();
    if (warp == 0) L2_MARK(10);

    // ---- 2c. down rows of this CTA for every member -> y / ys ----------------
    for (int i = nA + ((warp - nA % nw) % nw + nw) % nw; i < nA + nB && warp < nw; i += nw) {
        const int s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        const int row0 = P.b0 + (i - nA) * rows_b, nr = min(rows_b, P.b1 - row0);
        const char *s0 = routed ? LC.dsrc[u] : a.shared_down;
        const uint8_t *rows = stage_area + static_cast<size_t>(s) * a.stage_bytes +
                              ((reinterpret_cast<uintptr_t>(s0) + static_cast<uint64_t>(row0) * a.dn.row_bytes) & 15u);
        consume_tile<TB, ACT_CPU, 1, 1, 32>(a.dn, C, rows, rows, nr, u, U, row0, act_area, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    consumer_sync();          // the CTA's y stores, ordered before each warp's release below
    if (warp == 0) L2_MARK(11);

    // ---- 2d. arrivals per (token, row block); the CTA completing a block sums
    //      it: picks in order, then the shared expert --------------------------
    if (run && P.b1 > P.b0 && !epm) {
        const int RB = LAYER2_RB;
        const int rb0 = P.b0 / RB, nblk = (P.b1 - 1) / RB - rb0 + 1;
        for (int pair = warp; pair < nm * nblk; pair += PW) {
            const int m = pair / nblk, b = rb0 + pair % nblk;
            const int t = routed ? C.gmem[C.goff[u] + m] / k : m;
            const int lo = b * RB, hi = min(H, lo + RB);
            const uint32_t mine = static_cast<uint32_t>(min(P.b1, hi) - max(P.b0, lo));
            uint32_t old = 0;
            if (lane == 0) old = atom_add_acq_rel_gpu(&a.rowcnt[t * a.n_rb + b], mine);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old + mine != static_cast<uint32_t>(hi - lo) * static_cast<uint32_t>(k + hs)) continue;
            __syncwarp();
            const float *y = a.dn.dst + static_cast<int64_t>(t) * a.dn.stride_col_dst;
            for (int r = lo + lane; r < hi; r += 32) {
                float acc = 0.f;
                for (int p = 0; p < k; ++p) {
                    const float v = __fmul_rn(__ldcg(y + static_cast<int64_t>(p) * a.dn.stride_channel_dst + r), LC.wt[t * k + p]);
                    acc = p == 0 ? v : __fadd_rn(acc, v);
                }
                if (has_shared) acc = __fadd_rn(acc, __ldcg(a.dn.shared_dst + static_cast<int64_t>(t) * a.dn.shared_stride_col_dst + r));
                a.out[static_cast<int64_t>(t) * H + r] = acc;
            }
            if (lane == 0) atomicExch(&a.rowcnt[t * a.n_rb + b], 0u);
        }
    }
    if (epm) {
        // Expert-parallel: every routed row goes home -- token t lives on GPU
        // t -- as row p of its yhome (tagged words stored over NVLink); the
        // shared expert's rows go to row k of this GPU's own yhome. CTA c <
        // n_rb of every GPU then sums rows [64 c, 64 c + 64) of its own token:
        // each row's words polled until they carry this call's tag, picks in
        // order, then the shared expert. No fence or counter is needed.
        const EpDecodeLayout &Ly = a.ep.lay;
        const int RB = LAYER2_RB;
        const uint32_t etag = LC.xep + 1u;
        if (run && P.b1 > P.b0) {
            for (int m = 0; m < nm; ++m) {
                const float *src;
                uint64_t *dst;
                if (routed) {
                    const int e = C.gmem[C.goff[u] + m], t = e / k, p = e % k;
                    src = a.dn.dst + static_cast<int64_t>(t) * a.dn.stride_col_dst +
                          static_cast<int64_t>(p) * a.dn.stride_channel_dst;
                    dst = reinterpret_cast<uint64_t *>(a.ep.peer[t] + Ly.yhome) + static_cast<int64_t>(p) * H;
                } else {
                    src = a.dn.shared_dst + static_cast<int64_t>(m) * a.dn.shared_stride_col_dst;
                    dst = reinterpret_cast<uint64_t *>(a.ep.peer[me] + Ly.yhome) + static_cast<int64_t>(k) * H;
                }
                for (int r = P.b0 + tid; r < P.b1; r += PW * 32) st_relaxed_sys_u64(dst + r, tagged(__ldcg(src + r), etag));
            }
        }
        if (warp == 0) L2_MARK(19);
        if (bid < a.n_rb) {
            const int lo = bid * RB, hi = min(H, lo + RB);
            const uint64_t *yh = reinterpret_cast<const uint64_t *>(a.ep.peer[me] + Ly.yhome);
            const uint64_t t0 = clock64(), lim = timeout_cycles(a.ep_timeout_ns);
            auto take = [&](int p, int r) -> float {
                uint64_t w = ld_relaxed_sys_u64(yh + static_cast<int64_t>(p) * H + r);
                while (static_cast<uint32_t>(w >> 32) != etag) {
                    if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                        set_error(a.err, DERR_TIMEOUT_FULL);
                        break;
                    }
                    w = ld_relaxed_sys_u64(yh + static_cast<int64_t>(p) * H + r);
                }
                return __uint_as_float(static_cast<uint32_t>(w));
            };
            for (int r = lo + tid; r < hi; r += PW * 32) {
                float acc = 0.f;
                for (int p = 0; p < k; ++p) {
                    const float v = __fmul_rn(take(p, r), LC.wt[me * k + p]);
                    acc = p == 0 ? v : __fadd_rn(acc, v);
                }
                if (has_shared) acc = __fadd_rn(acc, take(k, r));
                a.out[r] = acc;
            }
            if (warp == 0) L2_MARK(20);
        }
    }

#ifdef MOE_LAYER2_TRACE
    consumer_sync();
    if (warp == 0) L2_MARK(12);
    if (tid == 0) g_layer2_trace[blockIdx.x * 64 + 31] = u;
#endif
    // ---- the last CTA to finish advances the epoch (every tagged read of this
    //      launch is done) ------------------------------------------------------
    if (tid == 0 && atomicAdd(&a.gbar[1], 1u) == gridDim.x - 1) {
        atomicExch(&a.gbar[1], 0u);
        atomicAdd(&a.gbar[0], 1u);
        if (epm) atomicAdd(reinterpret_cast<uint32_t *>(a.ep.peer[me] + a.ep.lay.epoch), 1u);
    }
}

}  // namespace moe
