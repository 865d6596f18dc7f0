// moe_layer.cuh -- one MoE layer of decode tokens in ONE kernel launch.
//
// The reference runs a MoE layer as separate graph nodes around its GEMV
// (routing, MUL_MAT_ID gate/up with the fused GLU, MUL_MAT_ID down, weighted
// sum; kernels/moe-cache.cu:72-291 is the GEMV of the two MUL_MAT_ID nodes).
// At batch 1 each of those launches moves a few MB, so launch latency and
// per-launch ramp-up dominate on a B200. This kernel does the whole layer in
// one cooperative launch of one CTA per SM:
//   1. the producer warp of every CTA routes (same bits as the routing
//      kernel), groups the picks and plans the CTA's tiles while the consumer
//      warps quantize the layer input;
//   2. the producer streams this CTA's gate/up rows (phase A: a contiguous
//      share of the (experts + shared) x F row space) and then its down rows
//      (phase B: output rows [h0, h1) of EVERY routed expert and of the
//      shared expert) through one shared-memory ring; phase B's weights do
//      not depend on phase A's results, so they stream in while phase A
//      computes;
//   3. consumer warps run phase A (fused gate/up + GLU), writing h also as
//      (value, launch tag) pairs; they then take h from the other CTAs block
//      by block as soon as a block's tags are this launch's (no grid
//      barrier), run phase B (down rows, writing y) and combine their own
//      output rows -- a CTA owns rows [h0, h1) of every pick, so the weighted
//      sum needs no exchange at all.
// Arithmetic per row is the GEMV's (consume_tile), so results match the
// multi-kernel path bit for bit. The launch tag is epoch + 1, where the
// epoch word (workspace) is advanced by the last CTA to finish.
#pragma once
#include "moe_gemv.cuh"
#include "moe_route.cuh"

namespace moe {

constexpr int LAYER_MAX_ENTRIES = 64;   // tokens x picks

// One expert tensor of the layer. tbl: the cache's tagged pointer table
// (bit 0 = host memory); null: expert e sits at dense + e * expert_bytes.
struct LayerTensor {
    const char *const *tbl;
    const char *dense;
    uint64_t expert_bytes;
    uint32_t *stamps;         // null: not a cache-registered tensor (no bookkeeping)
    int32_t cache_id, tma;
};

struct LayerArgs {
    // per-phase GEMV parameters: shapes, tile geometry, activation slots,
    // outputs and fusion (their table / routing fields are unused)
    GemvArgs gu, dn;
    LayerTensor up, gate, down;
    const char *shared_down;   // shared gate/up: gu.shared_up / gu.shared_gate
    int32_t tma_shared_down;
    const float *logits;
    int32_t n_tok, k, n_experts, norm_w;
    int32_t *ids_out;
    float *w_out, *out;
    uint32_t *stats;
    const uint32_t *clock;
    uint32_t log_cap;
    // h / hs exchange between CTAs: (value, tag) pairs, tag = launch epoch + 1
    uint64_t *h_tag, *hs_tag;
    uint32_t *gbar;            // [0] launch epoch, [1] finished CTAs (zero between launches)
    int32_t n_stages, rows_b;             // rows_b: rows of a phase-B tile
    uint32_t stage_bytes, ctrl_bytes, act_bytes;
    uint32_t part_bytes_b;                // a phase-B stage holds two tiles, one per half-warp
    int *err;
    uint64_t timeout_ns;
};

struct LayerCtrl {
    GemvCtrl g;
    const char *dsrc[LAYER_MAX_ENTRIES];
    uint8_t dkind[LAYER_MAX_ENTRIES], dhost[LAYER_MAX_ENTRIES];
    float wt[LAYER_MAX_ENTRIES];
    int32_t nA, nB, h0, h1, tpg;          // nB: phase-B tiles (two per stage)
    uint32_t tag;
};

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CONSUMER_WARPS * 32) : "memory");
}

template <int TA, int TB, int NMX>
__global__ void __launch_bounds__(GEMV_THREADS, 1) moe_layer_kernel(const __grid_constant__ LayerArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    LayerCtrl &LC = *reinterpret_cast<LayerCtrl *>(smem + 2 * GEMV_MAX_STAGES * 8);
    GemvCtrl &C = LC.g;
    uint8_t *act_area = smem + a.ctrl_bytes;
    uint8_t *stage_area = act_area + a.act_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.n_stages, k = a.k, n_tok = a.n_tok, N = n_tok * k;
    const int H = a.dn.nrows, F = a.gu.nrows;
    const bool has_shared = a.gu.shared_up != nullptr;

    // weight sources of an expert: tagged table entry or dense address
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
    auto x_of = [&](int e) { return C.x[e]; };
    auto resolve = [&](int u, int x) {
        src_of(a.up, x, C.usrc[u][0], C.ukind[u][0], C.uhost[u][0]);
        src_of(a.gate, x, C.usrc[u][1], C.ukind[u][1], C.uhost[u][1]);
        src_of(a.down, x, LC.dsrc[u], LC.dkind[u], LC.dhost[u]);
    };
    const int rpt = a.gu.rows_per_tile, rows_b = a.rows_b;
    // this CTA's tiles (one thread): phase A = its share of the (groups x F)
    // row space, phase B = rows [h0, h1) of every group
    // weighted: the split weighs each group by its members (C.wpre, made by
    // group_weight_prefix); unweighted: equal rows (one token: k distinct
    // picks of one member each, so the two agree in cost)
    auto plan_tiles = [&](int GA, bool weighted) {
        if (weighted) build_segments_weighted(C, GA, static_cast<uint32_t>(F), rpt, a.err);
        else build_segments(C, static_cast<uint32_t>(GA), static_cast<uint32_t>(F), rpt, a.err);
        const uint32_t G = gridDim.x, bid = blockIdx.x;
        const uint32_t q = static_cast<uint32_t>(H) / G, rem = static_cast<uint32_t>(H) % G;
        const int h0 = static_cast<int>(bid * q + (bid < rem ? bid : rem));
        const int h1 = h0 + static_cast<int>(q + (bid < rem ? 1u : 0u));
        const int tpg = (h1 - h0 + rows_b - 1) / rows_b;
        LC.h0 = h0;
        LC.h1 = h1;
        LC.tpg = tpg;
        LC.nA = C.n_tiles;
        LC.nB = GA * tpg;
    };

    // ---- 1. prologue --------------------------------------------------------
    // Up to 32 picks: the producer warp initialises the ring, selects token
    // 0's experts (the other tokens' picks come from consumer warps 1.. over
    // named barrier 2), groups the picks, and releases the consumers over
    // named barrier 3 (bar.arrive: it does not wait for them) to start
    // streaming. With one token the picks are distinct, so the tile plan only
    // needs their count: consumer warp 0 makes it meanwhile and hands it over
    // on named barrier 4. Consumer warps quantize x meanwhile. More picks:
    // everything over block barriers. Gating weights come later (3a).
    const int KA = a.gu.K;
    const bool small = N <= 32, one = n_tok == 1;
    const int PW = GEMV_CONSUMER_WARPS;   // producer warp
    const int GA1 = k + (has_shared ? 1 : 0);
    auto select = [&](int t) {
        route_select(a.logits + static_cast<int64_t>(t) * a.n_experts, a.n_experts, k, lane, &C.x[t * k]);
    };
    if (warp == PW) {
        for (int s = lane; s < S; s += 32) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
        if (lane == 0) {
            if (!(small && one)) C.fail = 0;   // else consumer warp 0 owns it until barrier 4
            LC.tag = ld_relaxed_u32(&a.gbar[0]) + 1u;
        }
        __syncwarp();
        if (small) {
            select(0);
            __syncwarp();
            if (one) {
                // k distinct picks: group u = pick u
                bool bad = false;
                if (lane < k) {
                    const int x = C.x[lane];
                    bad = x < 0 || x >= a.n_experts;
                    C.first[lane] = static_cast<int16_t>(lane);
                    C.uidx[lane] = static_cast<int16_t>(lane);
                    C.gmem[lane] = static_cast<int16_t>(lane);
                    C.goff[lane] = static_cast<int16_t>(lane);
                    C.uexp[lane] = x;
                    resolve(lane, x);
                }
                if (lane == 0) {
                    C.n_unique = k;
                    C.goff[k] = static_cast<int16_t>(k);
                }
                bad = __any_sync(0xffffffffu, bad);
                asm volatile("bar.sync 4, 64;" ::: "memory");    // the plan of warp 0
                if (bad && lane == 0) {
                    C.fail = 1;
                    set_error(a.err, DERR_BAD_ID);
                }
            } else {
                asm volatile("bar.sync 2, %0;" ::"r"(n_tok * 32) : "memory");
                build_groups_warp(C, N, a.n_experts, x_of, resolve, a.err, lane);
                __syncwarp();
                if (!C.fail) {
                    group_weight_prefix(C, C.n_unique, has_shared, n_tok, static_cast<uint32_t>(F), NMX, lane);
                    __syncwarp();
                    if (lane == 0) plan_tiles(C.n_unique + (has_shared ? 1 : 0), true);
                }
            }
            __syncwarp();
            asm volatile("bar.arrive 3, %0;" ::"r"(GEMV_THREADS) : "memory");
        }
    } else {
        if (small && one && warp == 0) {
            if (lane == 0) {
                C.fail = 0;
                plan_tiles(GA1, false);
            }
            __syncwarp();
            asm volatile("bar.arrive 4, 64;" ::: "memory");
        }
        // routers: tokens 1.. (small) or all tokens; the rest quantize x
        const bool router = small ? (warp >= 1 && warp < n_tok) : (warp < n_tok);
        if (router) {
            select(warp);
            if (small) asm volatile("bar.arrive 2, %0;" ::"r"(n_tok * 32) : "memory");
        } else {
            const int sidx = small ? (warp == 0 ? 0 : warp - n_tok + 1) : warp - n_tok;
            const int nst = small ? GEMV_CONSUMER_WARPS + 1 - n_tok : GEMV_CONSUMER_WARPS - n_tok;
            constexpr int QA = is_kquant(TA) ? 256 : 32;
            const int nb = KA / QA;
            for (int job = sidx; job < n_tok * nb; job += nst) {
                const int t = job / nb, b = job % nb;
                stage_f32_block<TA>(reinterpret_cast<const float *>(a.gu.y) + static_cast<int64_t>(t) * a.gu.stride_col_y,
                                    act_area + static_cast<size_t>(t) * a.gu.slot_bytes, KA, b, lane);
            }
        }
        // phase-A activation slot of every entry: its token's x
        for (int e = tid; e < N; e += GEMV_CONSUMER_WARPS * 32) C.eslot[e] = static_cast<int16_t>(e / k);
        if (tid < n_tok) C.shslot[tid] = static_cast<int16_t>(tid);
    }
    if (small) {
        if (warp != PW) asm volatile("bar.sync 3, %0;" ::"r"(GEMV_THREADS) : "memory");
    } else {
        __syncthreads();
        build_groups(C, N, a.n_experts, x_of, resolve, a.err);   // ends with a block barrier
        if (warp == 0 && !C.fail) {
            group_weight_prefix(C, C.n_unique, has_shared, n_tok, static_cast<uint32_t>(F), NMX, lane);
            __syncwarp();
            if (lane == 0) plan_tiles(C.n_unique + (has_shared ? 1 : 0), true);
        }
        __syncthreads();
    }
    const int U = C.n_unique;
    const bool run = !C.fail;
    const int nA = run ? LC.nA : 0, nB = run ? LC.nB : 0, n_seg = C.n_seg;
    const int nI = (nB + 1) / 2;   // phase-B ring stages
    const int h0 = LC.h0, h1 = LC.h1, tpg = LC.tpg;
    const uint32_t tag = LC.tag;

    auto phase_b_tile = [&](int j, int &g, int &row0, int &nr) {
        g = j / tpg;
        row0 = h0 + (j - g * tpg) * rows_b;
        nr = (h1 - row0) < rows_b ? (h1 - row0) : rows_b;
    };

    if (warp == GEMV_CONSUMER_WARPS) {
        // =========================== producer warp ===========================
        produce_tiles(
            nA + nI, S, full, empty, stage_area, a.stage_bytes,
            [&](int i, TileSrc &ts) {
                int g;
                if (i < nA) {
                    segment_tile(C, n_seg, rpt, i, g, ts.row0[0], ts.nr[0]);
                    ts.row0[1] = ts.row0[0];
                    ts.nr[1] = ts.nr[0];
                    if (g < U) {
                        ts.src[0] = C.usrc[g][0];
                        ts.src[1] = C.usrc[g][1];
                        ts.kind[0] = C.ukind[g][0];
                        ts.kind[1] = C.ukind[g][1];
                    } else {
                        ts.src[0] = a.gu.shared_up;
                        ts.src[1] = a.gu.shared_gate;
                        ts.kind[0] = ts.kind[1] = a.gu.tma_shared ? 0 : 2;
                    }
                    ts.n_parts = 2;
                    ts.rb = a.gu.row_bytes;
                    ts.part_bytes = a.gu.part_bytes;
                } else {
                    // phase-B stage: tiles 2j and 2j + 1, one per half-warp
                    const int j = 2 * (i - nA);
                    ts.n_parts = j + 1 < nB ? 2 : 1;
                    for (int p = 0; p < 2; ++p) {
                        ts.src[p] = nullptr;
                        ts.kind[p] = 0;
                        ts.row0[p] = ts.nr[p] = 0;
                        if (p >= ts.n_parts) continue;
                        phase_b_tile(j + p, g, ts.row0[p], ts.nr[p]);
                        ts.src[p] = g < U ? LC.dsrc[g] : a.shared_down;
                        ts.kind[p] = g < U ? LC.dkind[g] : (a.tma_shared_down ? 0 : 2);
                    }
                    ts.rb = a.dn.row_bytes;
                    ts.part_bytes = a.part_bytes_b;
                }
            },
            a.timeout_ns, a.err, lane);
        return;
    }

    // ============================ consumer warps =============================
    // ---- gating weights (warp t: token t; needed only by the combine) and
    //      the reference kernel's bookkeeping (:163-198, warp 0 of the first
    //      CTA), while the first tiles are in flight --------------------------
    if (run && warp < n_tok) {
        route_weights(a.logits + static_cast<int64_t>(warp) * a.n_experts, a.n_experts, k, a.norm_w, lane,
                      &C.x[warp * k], &LC.wt[warp * k]);
        __syncwarp();
        if (blockIdx.x == 0 && lane < k) a.w_out[warp * k + lane] = LC.wt[warp * k + lane];
    }
    if (blockIdx.x == 0 && run && warp == 0) {
        const uint32_t clk = a.clock ? *a.clock : 0u;
        for (int e = lane; e < N; e += 32) {
            const int x = C.x[e], u = C.uidx[e];
            a.ids_out[e] = x;
            const LayerTensor *T[3] = {&a.up, &a.gate, &a.down};
            const uint8_t host[3] = {C.uhost[u][0], C.uhost[u][1], LC.dhost[u]};
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

    // ---- 3a. phase A: fused gate/up + GLU -> h, hs --------------------------
    // tile i -> warp i % nw in both phases (n_stages is a multiple of nw)
    const int nw = a.gu.n_tile_warps;
    for (int i = warp; i < nA && warp < nw; i += nw) {
        const int s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        int g, row0, nr;
        segment_tile(C, n_seg, rpt, i, g, row0, nr);
        const char *s0 = g < U ? C.usrc[g][0] : a.gu.shared_up;
        const char *s1 = g < U ? C.usrc[g][1] : a.gu.shared_gate;
        const uint8_t *stage = stage_area + static_cast<size_t>(s) * a.stage_bytes;
        const uint64_t off = static_cast<uint64_t>(row0) * a.gu.row_bytes;
        const uint8_t *up_rows = stage + ((reinterpret_cast<uintptr_t>(s0) + off) & 15u);
        const uint8_t *gate_rows = stage + a.gu.part_bytes + ((reinterpret_cast<uintptr_t>(s1) + off) & 15u);
        consume_tile<TA, ACT_CPU, NMX, 2>(a.gu, C, up_rows, gate_rows, nr, g, U, row0, act_area, lane, a.h_tag,
                                          a.hs_tag, tag);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // every warp is past phase A: the activation slot map can change
    consumer_sync();
    // phase-B activation slots: entry e -> slot e, the shared block of token
    // t -> slot N + t (its input is hs)
    for (int e = tid; e < N; e += GEMV_CONSUMER_WARPS * 32) C.eslot[e] = static_cast<int16_t>(e);
    if (tid < n_tok) C.shslot[tid] = static_cast<int16_t>(N + tid);
    consumer_sync();

    // ---- 3b. quantize h (and hs) for phase B. Other CTAs wrote them as
    //      (value, tag) pairs: a block is taken once all its tags are this
    //      launch's, so no grid barrier is needed. Each warp loads up to 4
    //      blocks before quantizing any, so their latencies overlap ---------
    const int KB = a.dn.K;
    if (run) {
        constexpr bool KQ = is_kquant(TB);
        constexpr int QB = KQ ? 256 : 32, NV = KQ ? 8 : 1, BATCH = 4;
        const int nb = KB / QB;
        const int njobs = (N + (has_shared ? n_tok : 0)) * nb;
        auto block_of = [&](int job) -> const uint64_t * {
            const int v = job / nb, b = job % nb;
            const uint64_t *base;
            if (v < N) {
                const int t = v / k, p = v % k;
                base = a.h_tag + static_cast<int64_t>(p) * a.dn.stride_channel_y + static_cast<int64_t>(t) * a.dn.stride_col_y;
            } else {
                base = a.hs_tag + static_cast<int64_t>(v - N) * a.dn.shared_y_stride_col;
            }
            return base + b * QB;
        };
        // this lane's values of a block; true when all carry this launch's tag
        auto load = [&](const uint64_t *xb, float (&v)[NV]) -> bool {
            uint64_t w[NV];
            if constexpr (KQ) {
                ld_relaxed_u64x2(xb + 4 * lane, w[0], w[1]);
                ld_relaxed_u64x2(xb + 4 * lane + 2, w[2], w[3]);
                ld_relaxed_u64x2(xb + 128 + 4 * lane, w[4], w[5]);
                ld_relaxed_u64x2(xb + 128 + 4 * lane + 2, w[6], w[7]);
            } else {
                uint64_t unused;
                ld_relaxed_u64x2(xb + (lane & ~1), w[0], unused);
                if (lane & 1) w[0] = unused;
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
        for (int base = warp; base < njobs; base += GEMV_CONSUMER_WARPS * BATCH) {
            float vals[BATCH][NV];
            bool ok[BATCH];
#pragma unroll
            for (int r = 0; r < BATCH; ++r) {
                const int job = base + r * GEMV_CONSUMER_WARPS;
                ok[r] = true;
                if (job < njobs) ok[r] = load(block_of(job), vals[r]);
            }
            // re-read every block that is not complete yet, all at once, so
            // each poll costs one round trip
            for (;;) {
                unsigned waiting = 0;
#pragma unroll
                for (int r = 0; r < BATCH; ++r) {
                    const int job = base + r * GEMV_CONSUMER_WARPS;
                    if (job < njobs && !__all_sync(0xffffffffu, ok[r])) waiting |= 1u << r;
                }
                if (!waiting) break;
                if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                    if (lane == 0) set_error(a.err, DERR_TIMEOUT_TAG);
                    break;
                }
#pragma unroll
                for (int r = 0; r < BATCH; ++r)
                    if ((waiting >> r) & 1u) ok[r] = load(block_of(base + r * GEMV_CONSUMER_WARPS), vals[r]);
            }
#pragma unroll
            for (int r = 0; r < BATCH; ++r) {
                const int job = base + r * GEMV_CONSUMER_WARPS;
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

    // ---- 3c. phase B: down rows [h0, h1) of every group -> y, ys; each
    //      half-warp takes one of its stage's two tiles --------------------
    for (int i = nA + ((warp - nA % nw) % nw + nw) % nw; i < nA + nI && warp < nw; i += nw) {
        const int s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        const int half = lane >> 4, j = 2 * (i - nA) + half;
        if (j < nB) {
            int g, row0, nr;
            phase_b_tile(j, g, row0, nr);
            const char *s0 = g < U ? LC.dsrc[g] : a.shared_down;
            const uint8_t *stage = stage_area + static_cast<size_t>(s) * a.stage_bytes + half * a.part_bytes_b;
            const uint8_t *rows =
                stage + ((reinterpret_cast<uintptr_t>(s0) + static_cast<uint64_t>(row0) * a.dn.row_bytes) & 15u);
            consume_tile<TB, ACT_CPU, NMX, 1, 16>(a.dn, C, rows, rows, nr, g, U, row0, act_area, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    consumer_sync();

    // ---- 3d. weighted sum of this CTA's output rows (pick order) ------------
    const int nh = run ? h1 - h0 : 0;
    for (int idx = tid; idx < n_tok * nh; idx += GEMV_CONSUMER_WARPS * 32) {
        const int t = idx / nh, r = h0 + idx % nh;
        float acc = 0.f;
        for (int p = 0; p < k; ++p) {
            const float v = __fmul_rn(a.dn.dst[p * a.dn.stride_channel_dst + t * a.dn.stride_col_dst + r], LC.wt[t * k + p]);
            acc = p == 0 ? v : __fadd_rn(acc, v);
        }
        if (has_shared) acc = __fadd_rn(acc, a.dn.shared_dst[t * a.dn.shared_stride_col_dst + r]);
        a.out[static_cast<int64_t>(t) * H + r] = acc;
    }

    // ---- the last CTA to finish advances the epoch: every CTA has read it
    //      and every tagged read of this launch is done ----------------------
    if (tid == 0 && atomicAdd(&a.gbar[1], 1u) == gridDim.x - 1) {
        atomicExch(&a.gbar[1], 0u);
        atomicAdd(&a.gbar[0], 1u);
    }
}

}  // namespace moe
