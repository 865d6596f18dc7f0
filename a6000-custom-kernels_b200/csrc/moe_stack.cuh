// moe_stack.cuh -- batch-1 MoE layers back to back in ONE persistent launch.
//
// Each layer of a decode step has the same shape, and a layer's router logits
// are an input of the launch, so which experts a layer reads is known before
// the layer before it has finished. This kernel uses that: the producer warp
// of every CTA routes layer l + 1 itself and streams its tiles into the ring
// while the consumers still work on layer l. When a layer's input arrives,
// its weights are already in shared memory (the ring holds about one layer of
// a CTA's share), and what is left on the critical path per layer is the
// arithmetic and the exchanges between CTAs. One launch for many layers also
// keeps the code warm in the instruction cache and removes the launch gaps.
//
// Per layer l (one token): the same static plan as moe_layer2_kernel at batch
// 1 (unit u = pick u, the shared expert = unit k, CTA groups fixed), the same
// picks and weights (route_select / route_weights: descending logit, ties to
// the lower id) and tiles. Three exchanges, all by 64-bit (value, tag) words
// (tag = launch epoch + 1 + l; relaxed stores and loads, a reader that sees
// the tag sees the value): the h rows of each unit among its CTAs; the down
// rows of every unit (ytag), summed per 32-row block in pick order by the
// warp that owns the block, which writes out_l (and x_next_l = x_l + out_l
// when asked) and x_l + out_l tagged into xtag; and xtag, whose blocks every
// warp of every CTA polls before it stages layer l + 1's input -- so the
// layers may form a chain.
//
// Ring: tile i of layer l has ring index (tiles of layers 0..l-1) + i and is
// consumed by warp (ring index) % nw. Routing: the producer writes layer j's
// picks, weights and expert sources into buffer j % 3 and arrives on
// rt_full[j % 3]; the consumers release the buffer (rt_empty) when layer j is
// done, so the producer runs at most two layers ahead. All waits are bounded.
// Results equal moe_b200_layer_decode per layer bit for bit.
//
// Mixed stacks (moe_stack_kernel<T_STACK_MIXED, T_STACK_MIXED>): every layer
// names its own gate/up type and down type among Q2_K, Q3_K, Q4_K and Q6_K
// (llama.cpp's quantization mixes give each layer's tensors their own
// types). The kernel dispatches on them per layer: the tile geometry of each
// type comes from StackArgs::gum / dnm, tiles per layer vary (the ring index
// of a layer's first tile is the running sum), the stages are sized for the
// largest type present. A row's dot product does not depend on the tile it
// lands in, so a mixed stack equals moe_b200_layer_decode layer by layer too.
#pragma once
#include "moe_layer2.cuh"

namespace moe {

// One layer of the stack (device memory, read by every CTA).
struct StackLayer {
    const char *up, *gate, *down;           // expert 0 of each expert tensor (HBM)
    const char *sh_up, *sh_gate, *sh_down;  // the shared expert (null when none)
    const float *x, *logits;                // the token's input [H] and router logits [E]
    float *out, *x_next;                    // output [H]; x_next = x + out when not null
    int32_t *ids_out;                       // [k] picks (may be null)
    float *w_out;                           // [k] gating weights (may be null)
    int32_t chained;                        // x is the previous layer's x_next
    int32_t ta, tb;                         // mixed stacks: type slots of gate/up and down
};

// Template tag of the mixed-type kernel and its type slots.
constexpr int T_STACK_MIXED = 1 << 20;
constexpr int STACK_MIX_TYPES = 4;
__host__ __device__ constexpr int stack_mix_type(int slot) {
    return slot == 0 ? T_Q2_K : slot == 1 ? T_Q3_K : slot == 2 ? T_Q4_K : T_Q6_K;
}
__host__ __device__ constexpr int stack_mix_slot(int type) {
    return type == T_Q2_K ? 0 : type == T_Q3_K ? 1 : type == T_Q4_K ? 2 : type == T_Q6_K ? 3 : -1;
}
template <int T> struct StackType { static constexpr int value = T; };
// fn(StackType<type of slot>{}): one instantiation of fn per slot
template <class Fn>
__device__ __forceinline__ void with_stack_type(int slot, Fn &&fn) {
    switch (slot) {
        case 0: fn(StackType<T_Q2_K>{}); break;
        case 1: fn(StackType<T_Q3_K>{}); break;
        case 2: fn(StackType<T_Q4_K>{}); break;
        default: fn(StackType<T_Q6_K>{}); break;
    }
}

constexpr int STACK_MAX_K = 32;
#ifndef STACK_POLL_NS
#define STACK_POLL_NS 100
#endif
constexpr int STACK_ROUTE_BUFS = 3;
#ifndef STACK_COMBINE_W
#define STACK_COMBINE_W 9        // terms a combining warp polls per round: top-8 + shared in one
#endif

// One layer's routing, written by the producer warp, read by the consumers.
struct StackRoute {
    const char *usrc[STACK_MAX_K][2];       // up, gate rows of pick q
    const char *dsrc[STACK_MAX_K];          // down rows of pick q
    int32_t gid[STACK_MAX_K];
    float wt[STACK_MAX_K];
    int32_t bad;                            // a pick outside [0, n_experts)
};

// Shared memory the stack kernel adds after the layer kernel's control block.
struct StackShared {
    uint64_t rt_full[STACK_ROUTE_BUFS], rt_empty[STACK_ROUTE_BUFS];
    StackRoute r[STACK_ROUTE_BUFS];
};

struct StackArgs {
    GemvArgs gu, dn;                        // geometry; h, hs, y, ys in the workspace
    const StackLayer *layers;
    int32_t n_layers, k, n_experts, norm_w;
    uint64_t eb_up, eb_gate, eb_down;       // bytes of one expert of each tensor
    int32_t tma, has_shared;                // every source 16-byte aligned (bulk copies)
    uint64_t *h_tag, *hs_tag;
    uint64_t *ytag, *ytag_s;                // down rows as (value, tag): [k][ysc] routed, [H] shared
    int64_t ysc;
    uint64_t *xtag;                         // [2][H]: x_l + out_l as (value, tag), by layer parity
    uint32_t *gbar;                         // [0] epoch, [1] finished CTAs
    int32_t n_rb;
    int32_t n_stages, n_tile_warps;
    uint32_t stage_bytes, ctrl_bytes, act_bytes;
    uint32_t route_off;                     // byte offset of StackShared in shared memory
    int *err;
    uint64_t timeout_ns;
    GemvArgs gum[STACK_MIX_TYPES], dnm[STACK_MIX_TYPES];   // mixed stacks: gu / dn per type slot
};

// Tile geometry of one layer of the stack.
struct StackGeo {
    int ta, tb;                             // type slots (mixed stacks)
    int rpt, rows_b, nA, nB;                // rows per tile, tiles of each phase (this CTA)
    uint32_t rba, rbb, part_a;              // row bytes of gate/up and down, gate/up part size
};

// load_tagged_block for data this GPU's CTAs exchange (GPU scope)
template <bool KQ>
__device__ __forceinline__ bool load_tagged_block_gpu(const uint64_t *xb, uint32_t tag, int lane,
                                                      float (&v)[KQ ? 8 : 1]) {
    constexpr int NV = KQ ? 8 : 1;
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
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Optional timeline (built with -DMOE_LAYER2_TRACE): SM clock marks (64 per
// CTA) taken at one layer of the stack (MOE_STACK_TRACE_LAYER).
#ifdef MOE_LAYER2_TRACE
#ifndef MOE_STACK_TRACE_LAYER
#define MOE_STACK_TRACE_LAYER 20
#endif
#define ST_MARK(l, i)                                                                         \
    do {                                                                                      \
        if ((l) == MOE_STACK_TRACE_LAYER && lane == 0) g_layer2_trace[blockIdx.x * 64 + (i)] = clock64(); \
    } while (0)
#else
#define ST_MARK(l, i) do {} while (0)
#endif

template <int TA, int TB>
__global__ void __launch_bounds__(GEMV_THREADS, 1) moe_stack_kernel(const __grid_constant__ StackArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    Layer2Ctrl &LC = *reinterpret_cast<Layer2Ctrl *>(smem + 2 * GEMV_MAX_STAGES * 8);
    GemvCtrl &C = LC.g;
    StackShared &SS = *reinterpret_cast<StackShared *>(smem + a.route_off);
    uint8_t *act_area = smem + a.ctrl_bytes;
    uint8_t *stage_area = act_area + a.act_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.n_stages, k = a.k, E = a.n_experts, L = a.n_layers;
    const int H = a.dn.nrows, F = a.gu.nrows, KA = a.gu.K, KB = a.dn.K;
    const int hs = a.has_shared ? 1 : 0;
    const int G = gridDim.x, bid = blockIdx.x;
    const int rpt = a.gu.rows_per_tile, rows_b = a.dn.rows_per_tile;
    const int nw = a.n_tile_warps;
    constexpr int PW = GEMV_CONSUMER_WARPS;            // the producer warp
    const UnitPlan P = unit_plan(k + hs, nullptr, G, bid, F, H, rpt, rows_b);
    const bool shared_cta = hs && P.u == k;            // the shared expert's rows
    const uint8_t kind = a.tma ? 0 : 2;
    constexpr bool MIX = TA == T_STACK_MIXED;
    // this CTA's tiles of a layer (rows a0..a1 and b0..b1 do not depend on the type)
    auto geo_of = [&](const StackLayer &Lr) {
        StackGeo g;
        if constexpr (MIX) {
            g.ta = Lr.ta;
            g.tb = Lr.tb;
            const GemvArgs &ga = a.gum[g.ta], &gb = a.dnm[g.tb];
            g.rpt = ga.rows_per_tile;
            g.rows_b = gb.rows_per_tile;
            g.rba = ga.row_bytes;
            g.rbb = gb.row_bytes;
            g.part_a = ga.part_bytes;
            g.nA = (P.a1 - P.a0 + g.rpt - 1) / g.rpt;
            g.nB = (P.b1 - P.b0 + g.rows_b - 1) / g.rows_b;
        } else {
            g.ta = g.tb = 0;
            g.rpt = rpt;
            g.rows_b = rows_b;
            g.rba = a.gu.row_bytes;
            g.rbb = a.dn.row_bytes;
            g.part_a = a.gu.part_bytes;
            g.nA = P.nA;
            g.nB = P.nB;
        }
        return g;
    };

    if (warp == PW) {
        // ============================ producer warp ===========================
        for (int s = lane; s < S; s += 32) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        if (lane < STACK_ROUTE_BUFS) {
            mbar_init(&SS.rt_full[lane], 1);
            mbar_init(&SS.rt_empty[lane], 1);
        }
        fence_mbar_init();
        __syncwarp();
        asm volatile("bar.arrive 3, %0;" ::"r"(GEMV_THREADS) : "memory");

        // layer j's picks, weights and sources into buffer j % 3 (false: stop)
        auto route_layer = [&](int j) -> bool {
            const int b = j % STACK_ROUTE_BUFS;
            if (j >= STACK_ROUTE_BUFS &&
                !mbar_wait_sleep(&SS.rt_empty[b], static_cast<uint32_t>((j / STACK_ROUTE_BUFS - 1) & 1), a.timeout_ns)) {
                if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
                return false;
            }
            StackRoute &R = SS.r[b];
            const StackLayer &Lr = a.layers[j];
            route_select(Lr.logits, E, k, lane, R.gid);
            __syncwarp();
            const int x = lane < k ? R.gid[lane] : 0;
            const bool bad = __any_sync(0xffffffffu, x < 0 || x >= E);
            if (!bad) {
                route_weights(Lr.logits, E, k, a.norm_w, lane, R.gid, R.wt);
                // contiguous experts: a mixed layer's strides follow from its types
                uint64_t eb_up = a.eb_up, eb_gate = a.eb_gate, eb_down = a.eb_down;
                if constexpr (MIX) {
                    eb_up = eb_gate = static_cast<uint64_t>(F) * a.gum[Lr.ta].row_bytes;
                    eb_down = static_cast<uint64_t>(H) * a.dnm[Lr.tb].row_bytes;
                }
                if (lane < k) {
                    R.usrc[lane][0] = Lr.up + static_cast<uint64_t>(x) * eb_up;
                    R.usrc[lane][1] = Lr.gate + static_cast<uint64_t>(x) * eb_gate;
                    R.dsrc[lane] = Lr.down + static_cast<uint64_t>(x) * eb_down;
                    if (bid == 0 && Lr.ids_out) Lr.ids_out[lane] = x;
                    if (bid == 0 && Lr.w_out) Lr.w_out[lane] = R.wt[lane];
                }
            }
            if (lane == 0) R.bad = bad ? 1 : 0;   // reported by the consumers when they reach layer j
            __syncwarp();
            if (lane == 0) mbar_arrive(&SS.rt_full[b]);   // release: buffer b holds layer j
            return !bad;
        };
        // tile i of layer l (phase A: up + gate rows, then phase B: down rows)
        auto describe = [&](int l, const StackGeo &Gl, int i, TileSrc &ts) {
            const StackLayer &Lr = a.layers[l];
            const StackRoute &R = SS.r[l % STACK_ROUTE_BUFS];
            if (i < Gl.nA) {
                ts.row0[0] = ts.row0[1] = P.a0 + i * Gl.rpt;
                ts.nr[0] = ts.nr[1] = min(Gl.rpt, P.a1 - ts.row0[0]);
                ts.src[0] = shared_cta ? Lr.sh_up : R.usrc[P.u][0];
                ts.src[1] = shared_cta ? Lr.sh_gate : R.usrc[P.u][1];
                ts.kind[0] = ts.kind[1] = kind;
                ts.n_parts = 2;
                ts.rb = Gl.rba;
                ts.part_bytes = Gl.part_a;
            } else {
                const int jb = i - Gl.nA;
                ts.row0[0] = ts.row0[1] = P.b0 + jb * Gl.rows_b;
                ts.nr[0] = ts.nr[1] = min(Gl.rows_b, P.b1 - ts.row0[0]);
                ts.src[0] = ts.src[1] = shared_cta ? Lr.sh_down : R.dsrc[P.u];
                ts.kind[0] = ts.kind[1] = kind;
                ts.n_parts = 1;
                ts.rb = Gl.rbb;
                ts.part_bytes = a.stage_bytes;
            }
        };
        // stream: A(0) [route 1] B(0) A(1) [route 2] B(1) ... -- layer l + 1
        // is routed while layer l's down tiles wait for free stages
        int end = 0;   // ring indexes [0, end) issued
        if (route_layer(0)) {
            int g0 = 0;    // ring index of layer l's first tile
            for (int l = 0; l < L; ++l) {
                if (ld_relaxed_u32(reinterpret_cast<const uint32_t *>(a.err))) break;
                const StackGeo Gl = geo_of(a.layers[l]);
                ST_MARK(l, 7);
                int n = produce_tiles(Gl.nA, S, full, empty, stage_area, a.stage_bytes,
                                      [&](int i, TileSrc &ts) { describe(l, Gl, i, ts); }, a.timeout_ns, a.err, lane,
                                      g0, false);
                end = g0 + n;
                if (n < Gl.nA) break;
                ST_MARK(l, 8);
                const bool next = l + 1 < L ? route_layer(l + 1) : true;
                ST_MARK(l, 9);
                n = produce_tiles(Gl.nB, S, full, empty, stage_area, a.stage_bytes,
                                  [&](int i, TileSrc &ts) { describe(l, Gl, Gl.nA + i, ts); }, a.timeout_ns, a.err,
                                  lane, g0 + Gl.nA, false);
                end = g0 + Gl.nA + n;
                ST_MARK(l, 10);
                if (n < Gl.nB || !next) break;
                g0 += Gl.nA + Gl.nB;
            }
        }
        drain_tiles(end, S, full, a.timeout_ns, a.err, lane);   // nothing in flight at exit
        return;
    }
    // ============================ consumer warps =============================
    asm volatile("bar.sync 3, %0;" ::"r"(GEMV_THREADS) : "memory");   // the ring is initialised
    const uint32_t epoch0 = ld_relaxed_u32(&a.gbar[0]);
    // the groups are fixed: pick u = unit u, one member (entry u, token 0)
    if (tid < k) {
        C.first[tid] = static_cast<int16_t>(tid);
        C.uidx[tid] = static_cast<int16_t>(tid);
        C.gmem[tid] = static_cast<int16_t>(tid);
        C.goff[tid] = static_cast<int16_t>(tid);
        C.eslot[tid] = 0;
    }
    if (tid == 0) {
        C.n_unique = k;
        C.goff[k] = static_cast<int16_t>(k);
        C.shslot[0] = 0;
        C.fail = 0;
    }
#ifdef MOE_LAYER2_TRACE
    if (tid == 0)
        g_layer2_trace[bid * 64 + 63] = static_cast<unsigned long long>(S) | (static_cast<unsigned long long>(nw) << 8) |
                                        (static_cast<unsigned long long>(P.nA) << 16) |
                                        (static_cast<unsigned long long>(P.nB) << 24);
#endif
    // K-quant types (every mixed type) stage 256-value blocks, the others 32
    constexpr bool KQA = MIX || is_kquant(TA), KQB = MIX || is_kquant(TB);
    constexpr int QA = KQA ? 256 : 32;
    const int nbx = KA / QA;
    if (tid == 0) LC.halt = 0u;
    consumer_sync();
    // tile cursor of this warp (nw <= S, so one wrap per step at most); warps
    // past nw take no tiles
    int cg = warp < nw ? warp : 0x7fffffff, cs = warp < nw ? warp : 0;
    uint32_t cph = 0;
    int g0 = 0;    // ring index of layer l's first tile
    for (int l = 0; l < L; ++l) {
        const StackLayer &Lr = a.layers[l];
        const int rb = l % STACK_ROUTE_BUFS;
        const StackRoute &R = SS.r[rb];
        const uint32_t rpar = static_cast<uint32_t>((l / STACK_ROUTE_BUFS) & 1);
        const uint32_t tag = epoch0 + 1u + static_cast<uint32_t>(l);
        const StackGeo Gl = geo_of(Lr);
        const int nA = Gl.nA, nB = Gl.nB;
        if (warp == 0) ST_MARK(l, 0);
        // ---- layer l routed; its input staged. From layer 1 on, every value
        //      of x_l = x_{l-1} + out_{l-1} as layer l - 1's combiners tagged it
        //      (tag - 1): the layer starts only when layer l - 1 is complete,
        //      and a chained layer quantizes those values as its input -------
        if (tid == 0 && !mbar_wait_sleep(&SS.rt_full[rb], rpar, a.timeout_ns)) {
            set_error(a.err, DERR_TIMEOUT_FULL);
            LC.halt = 1u;
        }
        {
            constexpr bool KQ = KQA;
            const uint64_t *xin = a.xtag + static_cast<int64_t>(l & 1) * H;
            const bool from_tags = l > 0 && Lr.chained;
            const uint64_t t0 = clock64(), lim = timeout_cycles(a.timeout_ns);
            // every warp polls its own blocks of x_l directly (a pause between
            // rounds), so a block is staged one L2 round trip after its
            // combining warp wrote it (a watcher warp and a CTA barrier before
            // the loads cost a second round trip and the barrier per layer)
            // the activation layout is the gate/up type's
            auto stage_x = [&](auto tt) {
                constexpr int T = decltype(tt)::value;
                for (int b = warp; b < nbx; b += PW) {
                    float v[KQ ? 8 : 1];
                    if (l > 0) {
                        while (!__all_sync(0xffffffffu, load_tagged_block_gpu<KQ>(xin + b * QA, tag - 1u, lane, v))) {
                            if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                                if (lane == 0) {
                                    set_error(a.err, DERR_TIMEOUT_TAG);
                                    LC.halt = 1u;
                                }
                                break;
                            }
                            __nanosleep(2 * STACK_POLL_NS);
                        }
                    }
                    if (from_tags) {
                        int8_t *q = reinterpret_cast<int8_t *>(act_area);
                        int16_t *bs = reinterpret_cast<int16_t *>(act_area + KA);
                        float *sc = reinterpret_cast<float *>(act_area + KA + KA / 8);
                        if constexpr (KQ) quant_q8K_vals<T>(v, q, bs, sc, b, lane, KA / chunk_of<T>::CE);
                        else quant_q80_val<T>(v[0], q, bs, sc, b, lane, KA / chunk_of<T>::CE);
                    } else {
                        stage_f32_block<T, true>(Lr.x, act_area, KA, b, lane);
                    }
                }
            };
            if constexpr (MIX) with_stack_type(Gl.ta, stage_x);
            else stage_x(StackType<TA>{});
        }
        consumer_sync();
        if (warp == 0) ST_MARK(l, 2);
        if (LC.halt) break;
        // layer l - 1 is done in every consumer warp: its routing buffer is free
        if (l > 0 && tid == 0) mbar_arrive(&SS.rt_empty[(l - 1) % STACK_ROUTE_BUFS]);
        // thread 0 saw rt_full complete (acquiring the producer's writes) before
        // the barrier above, which orders it before every consumer's reads
        if (R.bad) {
            if (tid == 0) set_error(a.err, DERR_BAD_ID);
            break;
        }
        // ---- phase A: gate/up + GLU -> h, tagged copies -----------------------
        // this warp's tiles: the ring indexes = warp (mod nw), walked by the
        // cursor (cg, cs, cph) = (ring index, stage, phase parity)
        for (; cg < g0 + nA; cg += nw, cs += nw, cph ^= cs >= S ? 1u : 0u, cs -= cs >= S ? S : 0) {
            const int i = cg - g0, s = cs;
            if (i == warp && warp == 1) ST_MARK(l, 61);
            if (!mbar_wait_sleep(&full[s], cph, a.timeout_ns)) {
                if (lane == 0) {
                    set_error(a.err, DERR_TIMEOUT_FULL);
                    LC.halt = 1u;
                }
                break;
            }
            if (i == warp) ST_MARK(l, 12 + warp);
            const int row0 = P.a0 + i * Gl.rpt, nr = min(Gl.rpt, P.a1 - row0);
            const char *s0 = shared_cta ? Lr.sh_up : R.usrc[P.u][0];
            const char *s1 = shared_cta ? Lr.sh_gate : R.usrc[P.u][1];
            const uint8_t *stage = stage_area + static_cast<size_t>(s) * a.stage_bytes;
            const uint64_t off = static_cast<uint64_t>(row0) * Gl.rba;
            const uint8_t *up_rows = stage + ((reinterpret_cast<uintptr_t>(s0) + off) & 15u);
            const uint8_t *gate_rows = stage + Gl.part_a + ((reinterpret_cast<uintptr_t>(s1) + off) & 15u);
            auto tile_a = [&](auto tt) {
                constexpr int T = decltype(tt)::value;
                const GemvArgs &ga = MIX ? a.gum[stack_mix_slot(T) < 0 ? 0 : stack_mix_slot(T)] : a.gu;
                consume_tile<T, ACT_CPU, 1, 2>(ga, C, up_rows, gate_rows, nr, P.u, k, row0, act_area, lane, a.h_tag,
                                               a.hs_tag, tag);
            };
            if constexpr (MIX) with_stack_type(Gl.ta, tile_a);
            else tile_a(StackType<TA>{});
            if (i == warp) ST_MARK(l, 28 + warp);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (warp == 0) ST_MARK(l, 60);
        consumer_sync();
        if (warp == 0) ST_MARK(l, 3);
        // ---- the unit's h from the CTAs of its group, quantized for down ----
        {
            constexpr bool KQ = KQB;
            constexpr int QB = KQ ? 256 : 32;
            const int nb = KB / QB;
            const uint64_t *base = shared_cta ? a.hs_tag : a.h_tag + static_cast<int64_t>(P.u) * a.dn.stride_channel_y;
            const uint64_t t0 = clock64(), lim = timeout_cycles(a.timeout_ns);
            // quantized in the down type's layout
            auto stage_h = [&](auto tt) {
                constexpr int T = decltype(tt)::value;
                for (int b = warp; b < nb; b += PW) {
                    float v[KQ ? 8 : 1];
                    while (!__all_sync(0xffffffffu, load_tagged_block_gpu<KQ>(base + b * QB, tag, lane, v))) {
                        if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                            if (lane == 0) set_error(a.err, DERR_TIMEOUT_TAG);
                            break;
                        }
                        __nanosleep(STACK_POLL_NS);
                    }
                    int8_t *q = reinterpret_cast<int8_t *>(act_area);
                    int16_t *bs = reinterpret_cast<int16_t *>(act_area + KB);
                    float *sc = reinterpret_cast<float *>(act_area + KB + KB / 8);
                    if constexpr (KQ) quant_q8K_vals<T>(v, q, bs, sc, b, lane, KB / chunk_of<T>::CE);
                    else quant_q80_val<T>(v[0], q, bs, sc, b, lane, KB / chunk_of<T>::CE);
                }
            };
            if constexpr (MIX) with_stack_type(Gl.tb, stage_h);
            else stage_h(StackType<TB>{});
        }
        consumer_sync();
        if (warp == 0) ST_MARK(l, 4);
        // ---- phase B: down rows -> y / ys -------------------------------------
        for (; cg < g0 + nA + nB; cg += nw, cs += nw, cph ^= cs >= S ? 1u : 0u, cs -= cs >= S ? S : 0) {
            const int i = cg - g0, s = cs;
            if (i - nA < nw && warp == 1) ST_MARK(l, 11);
            if (!mbar_wait_sleep(&full[s], cph, a.timeout_ns)) {
                if (lane == 0) {
                    set_error(a.err, DERR_TIMEOUT_FULL);
                    LC.halt = 1u;
                }
                break;
            }
            if (i - nA < nw) ST_MARK(l, 44 + warp);
            if (i - nA < nw && warp == 1) ST_MARK(l, 62);
            const int row0 = P.b0 + (i - nA) * Gl.rows_b, nr = min(Gl.rows_b, P.b1 - row0);
            const char *s0 = shared_cta ? Lr.sh_down : R.dsrc[P.u];
            const uint8_t *rows = stage_area + static_cast<size_t>(s) * a.stage_bytes +
                                  ((reinterpret_cast<uintptr_t>(s0) + static_cast<uint64_t>(row0) * Gl.rbb) & 15u);
            auto tile_b = [&](auto tt) {
                constexpr int T = decltype(tt)::value;
                const GemvArgs &gb = MIX ? a.dnm[stack_mix_slot(T) < 0 ? 0 : stack_mix_slot(T)] : a.dn;
                consume_tile<T, ACT_CPU, 1, 1, 32>(gb, C, rows, rows, nr, P.u, k, row0, act_area, lane, a.ytag,
                                                   a.ytag_s, tag);
            };
            if constexpr (MIX) with_stack_type(Gl.tb, tile_b);
            else tile_b(StackType<TB>{});
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        consumer_sync();          // phase B has read the activation area; it may be restaged
        if (warp == 0) ST_MARK(l, 5);
        // ---- combine: CTA c sums the 32-row blocks b = c (mod G) (one lane per
        //      row) once every pick's rows and the shared expert's carry this
        //      layer's tag, in pick order; writes out (and x_next) and, tagged,
        //      x_l + out_l for layer l + 1 -----------------------------------------
        for (int j = PW - 1 - warp;; j += PW) {
            const int b = bid + j * G;
            if (b * 32 >= H) break;
            const int r = b * 32 + lane;
            const bool ok = r < H;
            const int np = k + hs;                       // the shared expert is term k
            const uint64_t t0 = clock64(), lim = timeout_cycles(a.timeout_ns);
            float acc = 0.f;
            bool fail = false;
            for (int p0 = 0; p0 < np && !fail; p0 += STACK_COMBINE_W) {
                uint64_t w[STACK_COMBINE_W];
                for (;;) {
                    bool got = true;
#pragma unroll
                    for (int q = 0; q < STACK_COMBINE_W; ++q) {
                        const int p = p0 + q;
                        const uint64_t *yp = p < k ? a.ytag + static_cast<int64_t>(p) * a.ysc : a.ytag_s;
                        w[q] = p < np && ok ? ld_relaxed_u64(yp + r) : tagged(0.f, tag);
                        got &= static_cast<uint32_t>(w[q] >> 32) == tag;
                    }
                    if (__all_sync(0xffffffffu, got)) break;
                    if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                        fail = true;
                        break;
                    }
                    __nanosleep(STACK_POLL_NS);
                }
#pragma unroll
                for (int q = 0; q < STACK_COMBINE_W; ++q) {
                    const int p = p0 + q;
                    if (p >= np || fail) break;
                    const float v = __uint_as_float(static_cast<uint32_t>(w[q]));
                    if (p < k) {
                        const float wv = __fmul_rn(v, R.wt[p]);
                        acc = p == 0 ? wv : __fadd_rn(acc, wv);
                    } else {
                        acc = __fadd_rn(acc, v);
                    }
                }
            }
            if (fail) {
                if (lane == 0) {
                    set_error(a.err, DERR_TIMEOUT_TAG);
                    LC.halt = 1u;
                }
                break;
            }
            if (ok) {
                // x_l: layer l - 1's tagged values for a chained layer, else the input
                const float x = l > 0 && Lr.chained
                                    ? __uint_as_float(static_cast<uint32_t>(
                                          ld_relaxed_u64(a.xtag + static_cast<int64_t>(l & 1) * H + r)))
                                    : __ldcg(Lr.x + r);
                const float xn = __fadd_rn(x, acc);
                Lr.out[r] = acc;
                if (Lr.x_next) Lr.x_next[r] = xn;
                st_relaxed_u64(a.xtag + static_cast<int64_t>((l + 1) & 1) * H + r, tagged(xn, tag));
            }
            ST_MARK(l, 40 + (warp & 3));
        }
        if (warp == 0) ST_MARK(l, 6);
        g0 += nA + nB;
    }
    // ---- the last CTA to finish advances the epoch past every layer's tag and
    //      clears the layer counter ---------------------------------------------
    if (tid == 0 && atomicAdd(&a.gbar[1], 1u) == gridDim.x - 1) {
        atomicExch(&a.gbar[1], 0u);
        atomicAdd(&a.gbar[0], static_cast<uint32_t>(L));
    }
}

}  // namespace moe
