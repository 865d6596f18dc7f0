// moe_layer.cuh -- one MoE layer of decode tokens in ONE kernel launch.
//
// The reference runs a MoE layer as separate graph nodes around its GEMV
// (routing, MUL_MAT_ID gate/up with the fused GLU, MUL_MAT_ID down, weighted
// sum; kernels/moe-cache.cu:72-291 is the GEMV of the two MUL_MAT_ID nodes).
// At batch 1 each of those launches moves a few MB, so launch latency and
// per-launch ramp-up dominate on a B200. This kernel does the whole layer in
// one cooperative launch of one CTA per SM:
//   1. every CTA routes every token itself (same bits as the routing kernel)
//      while its other warps quantize the layer input;
//   2. the producer warp streams this CTA's gate/up rows (phase A: a
//      contiguous share of the (experts + shared) x F row space) and then its
//      down rows (phase B: output rows [h0, h1) of EVERY routed expert and of
//      the shared expert) through one shared-memory ring; phase B's weights
//      do not depend on phase A's results, so they stream in while phase A
//      computes;
//   3. consumer warps run phase A (fused gate/up + GLU, writing h), meet the
//      other CTAs at one grid barrier, quantize h, run phase B (down rows,
//      writing y), and combine their own output rows -- a CTA owns rows
//      [h0, h1) of every pick, so the weighted sum needs no second barrier.
// Arithmetic per row is the GEMV's (consume_tile), so results match the
// multi-kernel path bit for bit.
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
    uint32_t *gbar;            // grid barrier words [2], zero between launches
    int32_t n_stages, rows_b;
    uint32_t stage_bytes, ctrl_bytes, act_bytes;
    int *err;
    uint64_t timeout_ns;
};

struct LayerCtrl {
    GemvCtrl g;
    const char *dsrc[LAYER_MAX_ENTRIES];
    uint8_t dkind[LAYER_MAX_ENTRIES], dhost[LAYER_MAX_ENTRIES];
    float wt[LAYER_MAX_ENTRIES];
    int32_t nA, nB, h0, h1, tpg;
};

// Grid-wide barrier for one thread per CTA of a co-resident grid. bar[0]
// counts arrivals, bar[1] departures; the last CTA to leave zeroes both, so
// the words are zero again when the launch ends. Gives up after ~timeout_ns.
__device__ __forceinline__ void grid_barrier(uint32_t *bar, uint64_t timeout_ns, int *err) {
    const uint32_t G = gridDim.x;
    __threadfence();
    atomicAdd(&bar[0], 1u);
    const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
    while (ld_acquire_gpu(&bar[0]) < G) {
        if (static_cast<uint64_t>(clock64()) - t0 > lim) { set_error(err, DERR_GRID_BARRIER); break; }
        __nanosleep(32);
    }
    __threadfence();
    if (atomicAdd(&bar[1], 1u) == G - 1) {
        atomicExch(&bar[0], 0u);
        atomicExch(&bar[1], 0u);
    }
}

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

    for (int s = tid; s < S; s += blockDim.x) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], 1);
    }
    if (tid < S) fence_mbar_init();
    if (tid == 0) C.fail = 0;

    // ---- 1. routing (warp t: token t) and phase-A activations (x) --------
    const int KA = a.gu.K;
    if (warp < n_tok) {
        route_token_warp(a.logits + static_cast<int64_t>(warp) * a.n_experts, a.n_experts, k, a.norm_w, lane,
                         &C.x[warp * k], &LC.wt[warp * k]);
    } else if (warp < GEMV_CONSUMER_WARPS) {
        constexpr int QA = is_kquant(TA) ? 256 : 32;
        const int nb = KA / QA;
        for (int job = warp - n_tok; job < n_tok * nb; job += GEMV_CONSUMER_WARPS - n_tok) {
            const int t = job / nb, b = job % nb;
            stage_f32_block<TA>(reinterpret_cast<const float *>(a.gu.y) + static_cast<int64_t>(t) * a.gu.stride_col_y,
                                act_area + static_cast<size_t>(t) * a.gu.slot_bytes, KA, b, lane);
        }
    }
    __syncthreads();

    // ---- 2. groups of distinct experts and their weight sources -----------
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
    build_groups(
        C, N, a.n_experts, [&](int e) { return C.x[e]; },
        [&](int u, int x) {
            src_of(a.up, x, C.usrc[u][0], C.ukind[u][0], C.uhost[u][0]);
            src_of(a.gate, x, C.usrc[u][1], C.ukind[u][1], C.uhost[u][1]);
            src_of(a.down, x, LC.dsrc[u], LC.dkind[u], LC.dhost[u]);
        },
        a.err);
    const int U = C.n_unique;
    const bool work = !C.fail;

    // ---- bookkeeping of the reference kernel, first CTA (:163-198) -------
    if (blockIdx.x == 0 && work) {
        const uint32_t clk = a.clock ? *a.clock : 0u;
        for (int e = tid; e < N; e += blockDim.x) {
            const int x = C.x[e], u = C.uidx[e];
            a.ids_out[e] = x;
            a.w_out[e] = LC.wt[e];
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

    // ---- this CTA's tiles --------------------------------------------------
    const int rpt = a.gu.rows_per_tile, rows_b = a.rows_b;
    if (tid == 0 && work) {
        const int GA = U + (has_shared ? 1 : 0);
        build_segments(C, static_cast<uint32_t>(GA), static_cast<uint32_t>(F), rpt, a.err);
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
    }
    // phase-A activation slot of every entry: its token's x
    for (int e = tid; e < N; e += blockDim.x) C.eslot[e] = static_cast<int16_t>(e / k);
    if (tid < n_tok) C.shslot[tid] = static_cast<int16_t>(tid);
    __syncthreads();
    const bool run = work && !C.fail;
    const int nA = run ? LC.nA : 0, nB = run ? LC.nB : 0, n_seg = C.n_seg;
    const int h0 = LC.h0, h1 = LC.h1, tpg = LC.tpg;

    auto phase_b_tile = [&](int j, int &g, int &row0, int &nr) {
        g = j / tpg;
        row0 = h0 + (j - g * tpg) * rows_b;
        nr = (h1 - row0) < rows_b ? (h1 - row0) : rows_b;
    };

    if (warp == GEMV_CONSUMER_WARPS) {
        // =========================== producer warp ===========================
        produce_tiles(
            nA + nB, S, full, empty, stage_area, a.stage_bytes, a.gu.part_bytes,
            [&](int i, TileSrc &ts) {
                int g;
                if (i < nA) {
                    segment_tile(C, n_seg, rpt, i, g, ts.row0, ts.nr);
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
                } else {
                    phase_b_tile(i - nA, g, ts.row0, ts.nr);
                    ts.src[0] = g < U ? LC.dsrc[g] : a.shared_down;
                    ts.kind[0] = g < U ? LC.dkind[g] : (a.tma_shared_down ? 0 : 2);
                    ts.src[1] = nullptr;
                    ts.kind[1] = 0;
                    ts.n_parts = 1;
                    ts.rb = a.dn.row_bytes;
                }
            },
            a.timeout_ns, a.err, lane);
        return;
    }

    // ============================ consumer warps =============================
    // ---- 3a. phase A: fused gate/up + GLU -> h, hs --------------------------
    for (int i = warp; i < nA; i += GEMV_CONSUMER_WARPS) {
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
        consume_tile<TA, ACT_CPU, NMX, 2>(a.gu, C, up_rows, gate_rows, nr, g, U, row0, act_area, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- grid barrier: every CTA's h is written -----------------------------
    consumer_sync();
    if (tid == 0) grid_barrier(a.gbar, a.timeout_ns, a.err);
    // phase-B activation slots: entry e -> slot e, the shared block of token
    // t -> slot N + t (its input is hs)
    for (int e = tid; e < N; e += GEMV_CONSUMER_WARPS * 32) C.eslot[e] = static_cast<int16_t>(e);
    if (tid < n_tok) C.shslot[tid] = static_cast<int16_t>(N + tid);
    consumer_sync();
    if (!run) return;

    // ---- 3b. quantize h (and hs) for phase B --------------------------------
    const int KB = a.dn.K;
    {
        constexpr int QB = is_kquant(TB) ? 256 : 32;
        const int nb = KB / QB;
        const int nkeys = N + (has_shared ? n_tok : 0);
        for (int job = warp; job < nkeys * nb; job += GEMV_CONSUMER_WARPS) {
            const int v = job / nb, b = job % nb;
            const float *src;
            if (v < N) {
                const int t = v / k, p = v % k;
                src = reinterpret_cast<const float *>(a.dn.y) + static_cast<int64_t>(p) * a.dn.stride_channel_y +
                      static_cast<int64_t>(t) * a.dn.stride_col_y;
            } else {
                src = reinterpret_cast<const float *>(a.dn.shared_y) + static_cast<int64_t>(v - N) * a.dn.shared_y_stride_col;
            }
            stage_f32_block<TB, true>(src, act_area + static_cast<size_t>(v) * a.dn.slot_bytes, KB, b, lane);
        }
    }
    consumer_sync();

    // ---- 3c. phase B: down rows [h0, h1) of every group -> y, ys ------------
    for (int j = warp; j < nB; j += GEMV_CONSUMER_WARPS) {
        const int i = nA + j, s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        int g, row0, nr;
        phase_b_tile(j, g, row0, nr);
        const char *s0 = g < U ? LC.dsrc[g] : a.shared_down;
        const uint8_t *stage = stage_area + static_cast<size_t>(s) * a.stage_bytes;
        const uint8_t *rows =
            stage + ((reinterpret_cast<uintptr_t>(s0) + static_cast<uint64_t>(row0) * a.dn.row_bytes) & 15u);
        consume_tile<TB, ACT_CPU, NMX, 1>(a.dn, C, rows, rows, nr, g, U, row0, act_area, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    consumer_sync();

    // ---- 3d. weighted sum of this CTA's output rows (pick order) ------------
    const int nh = h1 - h0;
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
}

}  // namespace moe
