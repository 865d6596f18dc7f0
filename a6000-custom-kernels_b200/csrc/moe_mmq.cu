// moe_mmq.cu -- prefill MUL_MAT_ID on tcgen05 (see moe_mmq.cuh): grouping of
// (token, pick) entries by expert, the B-tile gather and the grouped int8 GEMM.
#include <cstdio>

#include <cudaTypedefs.h>

#include "moe_aux.h"
#include "moe_mmq.cuh"

namespace moe {

// ---------------------------------------------------------------------------
// Grouping (one block): counts per expert, offsets, entries grouped by expert,
// and the tile prefix tile_off[e] = sum of ceil(count / NT) * row_blocks.
// Entry order inside an expert does not change any result.
// ---------------------------------------------------------------------------
__global__ void mmq_group_kernel(const int32_t *__restrict__ ids, int64_t ids_stride, int n_tok, int k, int E,
                                 int row_blocks, int32_t *cnt, int32_t *offsets, int32_t *cursor, int32_t *entries,
                                 int32_t *tile_off, int *err) {
    __shared__ int32_t warp_sum[32];
    __shared__ int32_t carry[2];
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += nth) cnt[e] = 0;
    __syncthreads();
    const int N = n_tok * k;
    for (int i = tid; i < N; i += nth) {
        const int t = i / k, p = i % k;
        const int x = ids[static_cast<int64_t>(t) * ids_stride + p];
        if (x < 0 || x >= E) {
            set_error(err, DERR_BAD_ID);
            continue;
        }
        atomicAdd(&cnt[x], 1);
    }
    __syncthreads();
    // two exclusive scans over the experts, nth at a time: offsets (entries)
    // and tile_off (tiles)
    if (tid == 0) { carry[0] = 0; carry[1] = 0; }
    __syncthreads();
    for (int base = 0; base < E; base += nth) {
        const int e = base + tid;
        const int c = e < E ? cnt[e] : 0;
        const int tl = e < E ? ((c + MMQ_NT - 1) / MMQ_NT) * row_blocks : 0;
        for (int which = 0; which < 2; ++which) {
            const int v = which == 0 ? c : tl;
            int incl = v;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += o;
            }
            if (lane == 31) warp_sum[warp] = incl;
            __syncthreads();
            if (warp == 0) {
                const int ws = lane < (nth + 31) / 32 ? warp_sum[lane] : 0;
                int wincl = ws;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int o = __shfl_up_sync(0xffffffffu, wincl, off);
                    if (lane >= off) wincl += o;
                }
                warp_sum[lane] = wincl - ws;   // exclusive prefix of warp sums
            }
            __syncthreads();
            const int excl = carry[which] + warp_sum[warp] + incl - v;
            if (e < E) {
                if (which == 0) { offsets[e] = excl; cursor[e] = excl; }
                else tile_off[e] = excl;
            }
            __syncthreads();
            if (tid == nth - 1) carry[which] = excl + v;
            __syncthreads();
        }
    }
    if (tid == 0) { offsets[E] = carry[0]; tile_off[E] = carry[1]; }
    __syncthreads();
    for (int i = tid; i < N; i += nth) {
        const int t = i / k, p = i % k;
        const int x = ids[static_cast<int64_t>(t) * ids_stride + p];
        if (x < 0 || x >= E) continue;
        entries[atomicAdd(&cursor[x], 1)] = i;
    }
}

// ---------------------------------------------------------------------------
// B tiles: per chunk (up to MMQ_NT entries of one expert) and super-block,
// with N = the chunk's token count rounded up to 16: the N float block scales
// (MMQ_BT_HEAD bytes), then the tokens' Q8_K quants in the MMA's K-major
// layout (16-byte chunk c of token j at c * 16 N + (j / 8) * 128 + (j % 8) * 16),
// chunk 16 = the 16 bsums' high parts (bsum >> 4, in [-127, 127]) and chunk
// 17 = their low nibbles (bsum & 15). Token slots past the chunk's count are
// zero.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) mmq_gather_q8K_kernel(const uint8_t *__restrict__ x8, int nsb, int E,
                                                             int row_blocks, int k, const int32_t *__restrict__ offsets,
                                                             const int32_t *__restrict__ entries,
                                                             const int32_t *__restrict__ tile_off,
                                                             uint8_t *__restrict__ btiles) {
    const int total = tile_off[E] / row_blocks * nsb;
    const int j = threadIdx.x >> 2, part = threadIdx.x & 3;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
        const int gc = w / nsb, sb = w - gc * nsb;
        // expert of chunk gc: the last e whose tile prefix is <= gc * row_blocks
        const int target = gc * row_blocks;
        int lo = 0, hi = E;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (tile_off[mid] <= target) lo = mid;
            else hi = mid;
        }
        const int chunk = gc - tile_off[lo] / row_blocks;
        const int ebeg = offsets[lo];
        const int nt = min(MMQ_NT, offsets[lo + 1] - ebeg - chunk * MMQ_NT);
        const int N = mmq_chunk_n(nt), CS = 16 * N;
        if (j >= N) continue;
        uint8_t *bt = btiles + static_cast<size_t>(w) * MMQ_BT_BYTES;
        uint8_t *tok = bt + MMQ_BT_HEAD + (j >> 3) * 128 + (j & 7) * 16;
        if (j < nt) {
            const int t = entries[ebeg + chunk * MMQ_NT + j] / k;
            const uint8_t *q8 = x8 + (static_cast<size_t>(t) * nsb + sb) * 292;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int kb = part * 4 + c;
                const uint32_t *q = reinterpret_cast<const uint32_t *>(q8 + 4 + 16 * kb);
                *reinterpret_cast<uint4 *>(tok + kb * CS) = make_uint4(q[0], q[1], q[2], q[3]);
            }
            if (part < 2) {
                uint32_t h[2] = {0u, 0u}, l[2] = {0u, 0u};
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const int bs = reinterpret_cast<const int16_t *>(q8 + 260)[8 * part + g];
                    h[g >> 2] |= (static_cast<uint32_t>(bs >> 4) & 0xFFu) << (8 * (g & 3));
                    l[g >> 2] |= (static_cast<uint32_t>(bs) & 0xFu) << (8 * (g & 3));
                }
                *reinterpret_cast<uint2 *>(tok + 16 * CS + 8 * part) = make_uint2(h[0], h[1]);
                *reinterpret_cast<uint2 *>(tok + 17 * CS + 8 * part) = make_uint2(l[0], l[1]);
            }
            if (part == 3) reinterpret_cast<float *>(bt)[j] = *reinterpret_cast<const float *>(q8);
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4 *>(tok + (part * 4 + c) * CS) = make_uint4(0, 0, 0, 0);
            if (part < 2) {
                *reinterpret_cast<uint2 *>(tok + 16 * CS + 8 * part) = make_uint2(0, 0);
                *reinterpret_cast<uint2 *>(tok + 17 * CS + 8 * part) = make_uint2(0, 0);
            }
            if (part == 3) reinterpret_cast<float *>(bt)[j] = 0.f;
        }
    }
}

// ---------------------------------------------------------------------------
// The grouped GEMM
// ---------------------------------------------------------------------------
template <int TYPE>
struct MmqType;
template <> struct MmqType<T_Q2_K> {
    static constexpr int BPB = 84;          // bytes per super-block
    static constexpr int NPLANE = 1;        // int8 planes of the folded weights
    static constexpr bool MINS = true;      // has the dmin * summs term
    static constexpr bool A_SIGNED = false; // folded weights sc * q in [0, 45]
};

// Shared-memory and TMEM layout of one CTA for weight type TYPE. TMEM
// columns: accumulator set s at s * 128 (isum planes from 0, summs at
// SUMMS_COL), A buffer b at 256 + b * 128 (quant planes: 64 columns each,
// then the mins: 8 columns).
template <int TYPE>
struct MmqLayout {
    using Ty = MmqType<TYPE>;
    static constexpr uint32_t SLOT = (Ty::BPB + 15) / 16 * 16 + 16;     // one row's window of one super-block
    static constexpr uint32_t CTRL = 8192;
    static constexpr int NB = 4;                                         // B-tile stages
    static constexpr uint32_t OFF_B = CTRL;
    static constexpr uint32_t OFF_P = (OFF_B + NB * MMQ_BT_BYTES + 127) / 128 * 128;
    static constexpr uint32_t STAGE = MMQ_M * SLOT;
    static constexpr int NP_FIT = static_cast<int>((227u * 1024u - OFF_P) / STAGE);
    static constexpr int NP = NP_FIT > 8 ? 8 : NP_FIT;                   // weight stages
    static constexpr uint32_t TOTAL = OFF_P + NP * STAGE;
    static constexpr uint32_t ACC_COLS = 128;                            // TMEM columns per accumulator set
    static constexpr uint32_t SUMMS_COL = Ty::NPLANE * MMQ_NT;           // summs plane within a set
    static constexpr uint32_t A_COL0 = 2 * ACC_COLS;                     // first A buffer
    static constexpr uint32_t A_COLS = 128;                              // TMEM columns per A buffer
    static constexpr uint32_t MINS_COL = Ty::NPLANE * 64;                // mins within an A buffer
    static_assert(NP >= 2, "at least two weight stages");
    static_assert(TOTAL <= 227u * 1024u, "shared memory budget");
    static_assert(SUMMS_COL + (Ty::MINS ? MMQ_NT : 0) <= ACC_COLS, "TMEM accumulator columns");
    static_assert(MINS_COL + (Ty::MINS ? 8 : 0) <= A_COLS && A_COL0 + 2 * A_COLS <= 512, "TMEM A columns");
    static_assert(SLOT % 16 == 0 && SLOT <= 256, "TMA box width");
};

// Warp roles: warps 0-7 finish the accumulators (warp w reads TMEM lanes
// 32 (w % 4) .. + 31, i.e. those weight rows, for token slices w / 4, w / 4 + 2),
// warps 8-15 unpack the weights (warp 8 + i: rows 32 (i % 4) + lane, elements
// 128 (i / 4) .. + 127 of each super-block), warp 16 loads, warps 17 and 18
// issue the MMAs of the even and the odd steps (an MMA instruction holds its
// issuing thread for ~100 cycles whatever N; two issuers overlap).
constexpr int MMQ_EPI_WARPS = 8;
constexpr int MMQ_UNP_WARPS = 8;
constexpr int MMQ_PROD_WARP = MMQ_EPI_WARPS + MMQ_UNP_WARPS;
constexpr int MMQ_MMA_WARP = MMQ_PROD_WARP + 1;   // and MMQ_MMA_WARP + 1
constexpr int MMQ_WS_THREADS = 32 * (MMQ_MMA_WARP + 2);
constexpr int MMQ_RING = 4;   // steps of row scales and token scales kept for the epilogue

struct MmqCtrl {   // fits MmqLayout::CTRL (static_assert in the kernel)
    uint64_t p_full[8], p_empty[8], b_full[4], b_empty[4];
    uint64_t mma_done[2];      // step g's MMAs complete (accumulator set g & 1 full, A buffer g & 1 free)
    uint64_t acc_empty[2];     // the epilogue has read accumulator set g & 1
    uint64_t a_ready[2];       // step g's A buffer g & 1 unpacked
    uint64_t s_full[MMQ_RING]; // step g's row and token scales written
    uint32_t tmem;
    int32_t abort;             // a wait timed out somewhere: every role stops
    alignas(16) float da[MMQ_RING][MMQ_NT];
    float2 rs[MMQ_RING][MMQ_M];
};

struct MmqTile {
    int e, rb, chunk, gchunk, ebeg, nt;
};

// Tile ti: expert (binary search of the tile prefix), row block, chunk of
// that expert, chunk index over all experts, first entry, token count.
// Consecutive tiles share the chunk and walk the row blocks.
__device__ __forceinline__ MmqTile mmq_tile(const MmqArgs &a, int ti, int row_blocks) {
    int lo = 0, hi = a.n_experts;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (a.tile_off[mid] <= ti) lo = mid;
        else hi = mid;
    }
    MmqTile T;
    T.e = lo;
    const int t0 = a.tile_off[lo];
    const int local = ti - t0;
    T.rb = local % row_blocks;
    T.chunk = local / row_blocks;
    T.gchunk = t0 / row_blocks + T.chunk;
    T.ebeg = a.offsets[lo];
    T.nt = min(MMQ_NT, a.offsets[lo + 1] - T.ebeg - T.chunk * MMQ_NT);
    return T;
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Bounded wait that also gives up once another role has aborted; a timeout
// aborts the block.
__device__ __forceinline__ bool mmq_wait(MmqCtrl &C, uint64_t *bar, uint32_t parity, const MmqArgs &a) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = clock64(), lim = timeout_cycles(a.timeout_ns);
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 2000u)) return true;
        if (*reinterpret_cast<volatile int32_t *>(&C.abort)) return false;
        if (static_cast<uint64_t>(clock64()) - t0 > lim) {
            *reinterpret_cast<volatile int32_t *>(&C.abort) = 1;
            set_error(a.err, DERR_TIMEOUT_FULL);
            return false;
        }
    }
}

// Half h of a Q2_K super-block (84 bytes at blk) of this thread's row:
// elements 128 h .. 128 h + 127 as folded int8 (sc * q) into A columns
// 32 h .. 32 h + 31 of the thread's TMEM lane at a_cols (element k in byte
// k % 4 of column k / 4); half 0 also writes the 16 mins as (16 m_g, m_g)
// into the 8 mins columns and returns the row's d and dmin.
__device__ __forceinline__ void unpack_q2K(const uint8_t *blk, uint32_t a_cols, int h, float &d, float &dm) {
    uint32_t sc4[4], qs[8], v[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc4[i] = ld_u32(blk + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) qs[i] = ld_u32(blk + 16 + 32 * h + 4 * i);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        // elements 16 kb .. 16 kb + 15 (kb = 8 h + c): plane c / 2 of quant
        // bytes 16 (c % 2) .. + 15 of the half's 32 bytes; one scale
        const int kb = 8 * h + c, plane = c >> 1, hb = c & 1;
        const uint32_t sc = (sc4[kb >> 2] >> (8 * (kb & 3))) & 0xFu;
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * c + i] = ((qs[4 * hb + i] >> (2 * plane)) & 0x03030303u) * sc;
    }
    tmem_st32(a_cols + 32 * h, v);
    if (h == 0) {
        const uint32_t m[8] = {sc4[0] & 0xF0F0F0F0u, sc4[1] & 0xF0F0F0F0u, sc4[2] & 0xF0F0F0F0u, sc4[3] & 0xF0F0F0F0u,
                               (sc4[0] >> 4) & 0x0F0F0F0Fu, (sc4[1] >> 4) & 0x0F0F0F0Fu, (sc4[2] >> 4) & 0x0F0F0F0Fu,
                               (sc4[3] >> 4) & 0x0F0F0F0Fu};
        tmem_st8(a_cols + MmqLayout<T_Q2_K>::MINS_COL, m);
        d = ld_half(blk + 80);
        dm = ld_half(blk + 82);
    }
}

// Instruction descriptor of kind::i8 with s32 accumulation: A unsigned or
// signed int8, B signed int8, both K-major
__host__ __device__ constexpr uint32_t mmq_idesc(bool a_signed, int N) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(MMQ_M >> 4) << 24);
}

template <int TYPE>
__global__ void __launch_bounds__(MMQ_WS_THREADS, 1) moe_mmq_kernel(const __grid_constant__ MmqArgs a) {
    using Lay = MmqLayout<TYPE>;
    using Ty = MmqType<TYPE>;
    static_assert(sizeof(MmqCtrl) <= Lay::CTRL, "control block too large");
    constexpr int BPB = Ty::BPB;
    extern __shared__ __align__(1024) uint8_t smem[];
    MmqCtrl &C = *reinterpret_cast<MmqCtrl *>(smem);
    uint8_t *B = smem + Lay::OFF_B;
    uint8_t *P = smem + Lay::OFF_P;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nsb = a.K / 256;
    const int row_blocks = a.nrows / MMQ_M;
    const int total = a.tile_off[a.n_experts];
    const int G = a.G, GR = MMQ_M / a.G;     // rows per tensor-map row; tensor-map rows per box

    if (tid == 0) {
        for (int s = 0; s < Lay::NP; ++s) {
            mbar_init(&C.p_full[s], 1);
            mbar_init(&C.p_empty[s], MMQ_UNP_WARPS);
        }
        for (int s = 0; s < Lay::NB; ++s) {
            mbar_init(&C.b_full[s], 1);
            mbar_init(&C.b_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&C.mma_done[s], 1);
            mbar_init(&C.acc_empty[s], MMQ_EPI_WARPS);
            mbar_init(&C.a_ready[s], MMQ_UNP_WARPS);
        }
        for (int s = 0; s < MMQ_RING; ++s) mbar_init(&C.s_full[s], MMQ_UNP_WARPS);
        C.abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&C.tmem)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = C.tmem;

    if (warp == MMQ_PROD_WARP) {
        // ---------------- producer: B tiles and weight rows ----------------------
        const uint64_t pol_w = l2_evict_first_policy(), pol_b = l2_evict_last_policy();
        uint32_t ps = 0, pph = 0, bs = 0, bph = 0, fills_p = 0, fills_b = 0;
        bool pok = true;
        for (int ti = blockIdx.x; ti < total && pok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(a, ti, row_blocks);
            const uint32_t bbytes = mmq_bt_bytes(mmq_chunk_n(T.nt));
            const int y0 = (T.e * a.nrows + T.rb * MMQ_M) / G;   // first tensor-map row of the tile
            for (int sb = 0; sb < nsb; ++sb) {
                bool w = lane == 0 ? mmq_wait(C, &C.b_empty[bs], bph ^ 1u, a) : true;
                if (!__shfl_sync(0xffffffffu, w, 0)) { pok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&C.b_full[bs], bbytes);
                    bulk_g2s(B + bs * MMQ_BT_BYTES, a.btiles + (static_cast<size_t>(T.gchunk) * nsb + sb) * MMQ_BT_BYTES,
                             bbytes, &C.b_full[bs], pol_b);
                }
                ++fills_b;
                if (++bs == Lay::NB) { bs = 0; bph ^= 1u; }

                w = lane == 0 ? mmq_wait(C, &C.p_empty[ps], pph ^ 1u, a) : true;
                if (!__shfl_sync(0xffffffffu, w, 0)) { pok = false; break; }
                // box j: the sb windows of rows G i + j, i < GR (16-byte aligned x)
                if (lane == 0) mbar_arrive_expect_tx(&C.p_full[ps], Lay::STAGE);
                __syncwarp();
                if (lane < G) {
                    const int x = (lane * static_cast<int>(a.row_bytes) + sb * BPB) & ~15;
                    tma_load_2d(P + ps * Lay::STAGE + lane * GR * Lay::SLOT, &a.rows, x, y0, &C.p_full[ps], pol_w);
                }
                ++fills_p;
                if (++ps == Lay::NP) { ps = 0; pph ^= 1u; }
            }
        }
        if (lane == 0) {
            // copies still in flight (only after an abort): wait for every
            // stage's last fill before the block may exit
            for (uint32_t s = 0; s < static_cast<uint32_t>(Lay::NP) && s < fills_p; ++s)
                mbar_wait_bounded(&C.p_full[s], ((fills_p - 1 - s) / Lay::NP) & 1u, a.timeout_ns);
            for (uint32_t s = 0; s < static_cast<uint32_t>(Lay::NB) && s < fills_b; ++s)
                mbar_wait_bounded(&C.b_full[s], ((fills_b - 1 - s) / Lay::NB) & 1u, a.timeout_ns);
        }
    } else if (warp >= MMQ_MMA_WARP) {
        // ---------------- MMA issuers (lane 0): steps g with g % 2 == warp parity ----
        const uint32_t par = static_cast<uint32_t>(warp - MMQ_MMA_WARP);
        if (lane == 0) {
            uint32_t g = 0, last = 0;
            bool ok = true, any = false;
            for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
                const MmqTile T = mmq_tile(a, ti, row_blocks);
                const int N = mmq_chunk_n(T.nt);
                const uint32_t bcs = 16u * N;   // B: bytes of one 16-byte K chunk over the N tokens
                const uint32_t idesc = mmq_idesc(Ty::A_SIGNED, N), idesc_m = mmq_idesc(false, N);
                for (int sb = 0; sb < nsb; ++sb, ++g) {
                    if ((g & 1u) != par) continue;
                    const uint32_t bs = g % Lay::NB, bph = (g / Lay::NB) & 1u;
                    // A buffer g & 1 unpacked, B tile landed, accumulator set
                    // g & 1 read by step g - 2's epilogue
                    ok = mmq_wait(C, &C.a_ready[par], (g >> 1) & 1u, a) && mmq_wait(C, &C.b_full[bs], bph, a) &&
                         (g < 2 || mmq_wait(C, &C.acc_empty[par], ((g - 2) >> 1) & 1u, a));
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t a0 = tmem + Lay::A_COL0 + par * Lay::A_COLS;
                    const uint32_t b0 = smem_u32(B + bs * MMQ_BT_BYTES) + MMQ_BT_HEAD;
                    const uint32_t d0 = tmem + par * Lay::ACC_COLS;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        umma_i8_ts(d0, a0 + 8 * kk, umma_desc(b0 + kk * 2 * bcs, bcs, 128), idesc, kk > 0 ? 1u : 0u);
                    if (Ty::MINS)   // summs = sum_g (16 m_g) hi_g + m_g lo_g
                        umma_i8_ts(d0 + Lay::SUMMS_COL, a0 + Lay::MINS_COL, umma_desc(b0 + 16 * bcs, bcs, 128), idesc_m, 0u);
                    umma_commit(&C.mma_done[par]);
                    umma_commit(&C.b_empty[bs]);
                    last = g;
                    any = true;
                }
            }
            if (any)   // this issuer's last MMAs before TMEM is freed
                mbar_wait_bounded(&C.mma_done[par], (last >> 1) & 1u, a.timeout_ns);
        }
    } else if (warp >= MMQ_EPI_WARPS) {
        // ---------------- unpack warps -------------------------------------------
        const int uw = warp - MMQ_EPI_WARPS;
        const int r = 32 * (uw & 3) + lane, h = uw >> 2;   // row, half of the super-block
        // row r's window in a weight stage: box r % G, line r / G
        const uint32_t slot_off = static_cast<uint32_t>((r % G) * GR + r / G) * Lay::SLOT;
        const uint32_t row_in_group = static_cast<uint32_t>(r % G) * a.row_bytes;
        uint32_t ps = 0, pph = 0, bs = 0, bph = 0, g = 0;
        bool ok = true;
        // this thread's TMEM lane (row r) in the A buffers
        const uint32_t a_lane = tmem + (static_cast<uint32_t>(32 * (uw & 3)) << 16) + Lay::A_COL0;
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
            for (int sb = 0; sb < nsb; ++sb, ++g) {
                // weight stage landed; A buffer g & 1 last read by step g - 2's MMAs
                ok = mmq_wait(C, &C.p_full[ps], pph, a) &&
                     (g < 2 || mmq_wait(C, &C.mma_done[g & 1u], ((g - 2) >> 1) & 1u, a));
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint8_t *slot = P + ps * Lay::STAGE + slot_off + ((row_in_group + static_cast<uint32_t>(sb) * BPB) & 15u);
                float d, dm;
                unpack_q2K(slot, a_lane + (g & 1u) * Lay::A_COLS, h, d, dm);
                if (h == 0) C.rs[g % MMQ_RING][r] = make_float2(d, dm);
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.p_empty[ps]);
                if (++ps == Lay::NP) { ps = 0; pph ^= 1u; }
                if (uw < 2) {   // rows 0-63 of half 0 copy the token scales
                    ok = mmq_wait(C, &C.b_full[bs], bph, a);
                    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                    C.da[g % MMQ_RING][r] = reinterpret_cast<const float *>(B + bs * MMQ_BT_BYTES)[r];
                }
                if (++bs == Lay::NB) { bs = 0; bph ^= 1u; }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&C.a_ready[g & 1u]);
                    mbar_arrive(&C.s_full[g % MMQ_RING]);
                }
            }
        }
    } else {
        // ---------------- epilogue warps -----------------------------------------
        const int r = 32 * (warp & 3) + lane, half = warp >> 2;   // row; token slices half, half + 2
        float acc[MMQ_NT / 2];
#pragma unroll
        for (int n = 0; n < MMQ_NT / 2; ++n) acc[n] = 0.f;
        uint32_t g = 0;
        bool ok = true;
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(a, ti, row_blocks);
            for (int sb = 0; sb < nsb; ++sb, ++g) {
                ok = mmq_wait(C, &C.s_full[g % MMQ_RING], (g / MMQ_RING) & 1u, a) &&
                     mmq_wait(C, &C.mma_done[g & 1u], (g >> 1) & 1u, a);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint32_t cols = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + (g & 1u) * Lay::ACC_COLS;
                const float2 rs = C.rs[g % MMQ_RING][r];
                const float *dav = C.da[g % MMQ_RING];
                // llama.cpp's sumf += (d_a d) * isum - (d_a dmin) * summs, per token
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int sl = half + 2 * q;
                    if (sl * 16 < T.nt) {
                        uint32_t S[16], M[16];
                        tmem_ld16(cols + sl * 16, S);
                        tmem_ld16(cols + Lay::SUMMS_COL + sl * 16, M);
                        tmem_wait_ld();
                        float dv[16];
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 t4 = *reinterpret_cast<const float4 *>(dav + sl * 16 + j);
                            dv[j] = t4.x; dv[j + 1] = t4.y; dv[j + 2] = t4.z; dv[j + 3] = t4.w;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float da = dv[j];
                            const float dall = __fmul_rn(da, rs.x), dmin = __fmul_rn(da, rs.y);
                            const float fi = small_int_to_float(static_cast<int>(S[j]));
                            const float fm = small_int_to_float(static_cast<int>(M[j]));
                            acc[q * 16 + j] = __fadd_rn(acc[q * 16 + j], __fsub_rn(__fmul_rn(dall, fi), __fmul_rn(dmin, fm)));
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.acc_empty[g & 1u]);
                if (sb == nsb - 1) {
                    const int row = T.rb * MMQ_M + r;
                    const int32_t *ent = a.entries + T.ebeg + T.chunk * MMQ_NT;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = (half + 2 * q) * 16 + j;
                            if (n < T.nt) a.dst[static_cast<int64_t>(ent[n]) * a.nrows + row] = acc[q * 16 + j];
                            acc[q * 16 + j] = 0.f;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u)
                     : "memory");
}

cudaError_t launch_mmq_group(const int32_t *ids, int64_t ids_stride, int n_tok, int k, int E, int row_blocks,
                             int32_t *cnt, int32_t *offsets, int32_t *cursor, int32_t *entries, int32_t *tile_off,
                             int *err, cudaStream_t st) {
    mmq_group_kernel<<<1, 1024, 0, st>>>(ids, ids_stride, n_tok, k, E, row_blocks, cnt, offsets, cursor, entries,
                                         tile_off, err);
    return cudaGetLastError();
}

cudaError_t launch_mmq_gather(const uint8_t *x8, int nsb, int E, int row_blocks, int k, const int32_t *offsets,
                              const int32_t *entries, const int32_t *tile_off, int64_t max_chunks, uint8_t *btiles,
                              cudaStream_t st) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t work = max_chunks * nsb;
    const int grid = static_cast<int>(work < 8 * n_sm ? (work > 0 ? work : 1) : 8 * n_sm);
    mmq_gather_q8K_kernel<<<grid, 256, 0, st>>>(x8, nsb, E, row_blocks, k, offsets, entries, tile_off, btiles);
    return cudaGetLastError();
}

bool mmq_supported(int type, int64_t K, int64_t nrows) {
    return type == T_Q2_K && K % 256 == 0 && nrows % MMQ_M == 0;
}

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Rows of the expert tensor as a 2-D uint8 tensor of G-row groups
// (G * row_bytes a multiple of 16), box {slot, 128 / G}
bool encode_rows_map(MmqArgs &a, uint32_t slot) {
    int G = 1;
    while ((static_cast<uint64_t>(G) * a.row_bytes) % 16 != 0) G *= 2;
    if (G > 16) return false;
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(G) * a.row_bytes,
                                static_cast<cuuint64_t>(a.n_experts) * a.nrows / G};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(G) * a.row_bytes};
    const cuuint32_t box[2] = {slot, static_cast<cuuint32_t>(MMQ_M / G)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&a.rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<char *>(a.dense), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    a.G = G;
    return r == CUDA_SUCCESS;
}

}  // namespace

int launch_mmq(int type, MmqArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    if (!mmq_supported(type, a.K, a.nrows)) {
        *why = "tensor-core prefill needs Q2_K, K % 256 == 0 and rows % 128 == 0";
        return -2;
    }
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;
    using Lay = MmqLayout<T_Q2_K>;
    if ((reinterpret_cast<uintptr_t>(a.dense) & 15u) != 0 || !encode_rows_map(a, Lay::SLOT)) {
        *why = "cannot describe the expert rows as a TMA tensor map";
        return -2;
    }
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -3;
    auto kern = moe_mmq_kernel<T_Q2_K>;
    if (!configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::TOTAL);
        if (e != cudaSuccess) { *cuda_err = e; *why = "cudaFuncSetAttribute"; return -3; }
        configured[dev] = true;
    }
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    kern<<<n_sm, MMQ_WS_THREADS, Lay::TOTAL, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { *cuda_err = e; *why = "moe_mmq_kernel launch"; return -3; }
    return 0;
}

}  // namespace moe
