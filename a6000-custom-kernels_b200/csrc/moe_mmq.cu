// moe_mmq.cu -- prefill MUL_MAT_ID on tcgen05 (see moe_mmq.cuh): grouping of
// (token, pick) entries by expert, the B-tile gather and the grouped int8 GEMM.
#include <cstdio>

#include <cudaTypedefs.h>

#include "moe_aux.h"
#include "moe_mmq.cuh"

namespace moe {

// ---------------------------------------------------------------------------
// Grouping (one block, counters in shared memory): the entries (tok * k +
// pick) grouped by expert, and the chunk table: an expert's entries form
// chunks of up to ntc, chunk c = {expert, first entry, token count}, chunks of
// an expert consecutive, *n_chunks their count. Entry order inside an expert
// does not change any result. With skip_empty, id -1 marks an empty slot
// (expert-parallel receive regions) and is left out without an error.
// ---------------------------------------------------------------------------
constexpr int MMQ_GROUP_REG = 8;   // ids kept in registers per thread (n_tok * k <= 8192)

__global__ void __launch_bounds__(1024) mmq_group_kernel(const int32_t *__restrict__ ids, int64_t ids_stride, int n_tok,
                                                         int k, int E, int ntc, int skip_empty, int32_t *entries,
                                                         int4 *chunks, int32_t *n_chunks, int *err) {
    extern __shared__ int32_t cnt[];   // [E] counts, then scatter cursors
    __shared__ int32_t warp_sum[32];
    __shared__ int32_t carry[2];
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += nth) cnt[e] = 0;
    if (tid == 0) { carry[0] = 0; carry[1] = 0; }
    __syncthreads();
    const int N = n_tok * k;
    const bool in_regs = N <= MMQ_GROUP_REG * nth;
    int xr[MMQ_GROUP_REG];
    auto id_of = [&](int i) {
        const int t = i / k, p = i - t * k;
        return ids[static_cast<int64_t>(t) * ids_stride + p];
    };
#pragma unroll
    for (int u = 0; u < MMQ_GROUP_REG; ++u) {
        const int i = tid + u * nth;
        xr[u] = (in_regs && i < N) ? id_of(i) : -1;
    }
    // warp-aggregated increments: one atomic per distinct expert in the warp
    auto count = [&](int x, bool valid) {
        const bool bad = valid && (x >= E || (x < 0 && !(skip_empty && x == -1)));   // -1: an empty slot
        if (bad) set_error(err, DERR_BAD_ID);
        const bool use = valid && !bad && x >= 0;
        const unsigned peers = __match_any_sync(0xffffffffu, use ? x : -1);
        if (use && lane == __ffs(peers) - 1) atomicAdd(&cnt[x], __popc(peers));
    };
    if (in_regs) {
#pragma unroll
        for (int u = 0; u < MMQ_GROUP_REG; ++u) count(xr[u], tid + u * nth < N);
    } else {
        for (int i0 = 0; i0 < N; i0 += nth) count(i0 + tid < N ? id_of(i0 + tid) : -1, i0 + tid < N);
    }
    __syncthreads();
    // two exclusive scans over the experts, nth at a time: first entries and
    // first chunks; the counts become the scatter cursors
    for (int base = 0; base < E; base += nth) {
        const int e = base + tid;
        const int c = e < E ? cnt[e] : 0;
        const int nc = (c + ntc - 1) / ntc;
        int excl_v[2];
        for (int which = 0; which < 2; ++which) {
            const int v = which == 0 ? c : nc;
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
            excl_v[which] = carry[which] + warp_sum[warp] + incl - v;
            __syncthreads();
            if (tid == nth - 1) carry[which] = excl_v[which] + v;
            __syncthreads();
        }
        if (e < E) {
            cnt[e] = excl_v[0];
            for (int q = 0; q < nc; ++q)
                chunks[excl_v[1] + q] = make_int4(e, excl_v[0] + q * ntc, min(ntc, c - q * ntc), q);
        }
    }
    if (tid == 0) *n_chunks = carry[1];
    __syncthreads();
    // warp-aggregated placement: the lowest lane of each expert's peers takes
    // a run of slots, the peers fill it in lane order
    auto place = [&](int i, int x, bool valid) {
        const bool use = valid && x >= 0 && x < E;
        const unsigned peers = __match_any_sync(0xffffffffu, use ? x : -1);
        const int leader = __ffs(peers) - 1;
        int base = 0;
        if (use && lane == leader) base = atomicAdd(&cnt[x], __popc(peers));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (use) entries[base + __popc(peers & ((1u << lane) - 1u))] = i;
    };
    if (in_regs) {
#pragma unroll
        for (int u = 0; u < MMQ_GROUP_REG; ++u) place(tid + u * nth, xr[u], tid + u * nth < N);
    } else {
        for (int i0 = 0; i0 < N; i0 += nth) place(i0 + tid, i0 + tid < N ? id_of(i0 + tid) : -1, i0 + tid < N);
    }
}

// ---------------------------------------------------------------------------
// B tiles: per chunk and super-block, with N = the chunk's token count
// rounded up to 16: the head (block scales, bsum pairs; MMQ_BT_HEAD bytes), then the
// tokens' Q8_K quants in the MMA's K-major layout (16-byte chunk c of token j
// at c * 16 N + (j / 8) * 128 + (j % 8) * 16), chunk 16 = the 16 bsums' high
// parts (bsum >> 4, in [-127, 127]) and chunk 17 = their low nibbles
// (bsum & 15); the head also holds the 8 sums of bsum pairs (one per 32
// values). Token slots past the chunk's count are zero. Copied from the
// tokens' Q8_K rows x8 (292-byte blocks), one warp per token slot for all its
// super-blocks.
// ---------------------------------------------------------------------------
constexpr int MMQ_GATHER_MAX_SB = 16;   // K <= 4096

__device__ __forceinline__ void mmq_gather_slot(const uint8_t *__restrict__ x8, int nsb, int k, int ntc,
                                                const int32_t *__restrict__ entries, const int4 *__restrict__ chunks,
                                                uint8_t *__restrict__ btiles, int wg, int lane) {
    const int gc = wg / ntc, j = wg - gc * ntc;   // chunk, token slot
    const int4 ch = chunks[gc];
    const int nt = ch.z, N = mmq_chunk_n(nt), CS = 16 * N;
    if (j >= N) return;
    const int t = j < nt ? entries[ch.y + j] / k : -1;
    const uint8_t *row = x8 + static_cast<size_t>(t < 0 ? 0 : t) * nsb * 292;
    // all super-blocks' loads first (nsb <= MMQ_GATHER_MAX_SB), then the stores
    uint32_t w0[MMQ_GATHER_MAX_SB], w1[MMQ_GATHER_MAX_SB], hl[MMQ_GATHER_MAX_SB];
    int bsv[MMQ_GATHER_MAX_SB];
    float d[MMQ_GATHER_MAX_SB];
#pragma unroll
    for (int sb = 0; sb < MMQ_GATHER_MAX_SB; ++sb) {
        w0[sb] = w1[sb] = hl[sb] = 0u;
        bsv[sb] = 0;
        d[sb] = 0.f;
        if (sb < nsb && t >= 0) {
            const uint8_t *blk = row + sb * 292;   // 4-byte aligned
            // quants 8 lane .. 8 lane + 7; lane 2 g: bsum g; lane 0: the scale
            w0[sb] = *reinterpret_cast<const uint32_t *>(blk + 4 + 8 * lane);
            w1[sb] = *reinterpret_cast<const uint32_t *>(blk + 8 + 8 * lane);
            const int bs = reinterpret_cast<const int16_t *>(blk + 260)[lane >> 1];
            hl[sb] = (static_cast<uint32_t>(bs >> 4) & 0xFFu) | ((static_cast<uint32_t>(bs) & 0xFu) << 8);
            bsv[sb] = bs;
            if (lane == 0) d[sb] = *reinterpret_cast<const float *>(blk);
        }
    }
#pragma unroll
    for (int sb = 0; sb < MMQ_GATHER_MAX_SB; ++sb) {
        if (sb < nsb) {
            uint8_t *bt = btiles + (static_cast<size_t>(gc) * nsb + sb) * MMQ_BT_BYTES;
            uint8_t *tok = bt + MMQ_BT_HEAD + (j >> 3) * 128 + (j & 7) * 16;
            *reinterpret_cast<uint2 *>(tok + (lane >> 1) * CS + 8 * (lane & 1)) = make_uint2(w0[sb], w1[sb]);
            if ((lane & 1) == 0) {
                tok[16 * CS + (lane >> 1)] = static_cast<uint8_t>(hl[sb] & 0xFFu);
                tok[17 * CS + (lane >> 1)] = static_cast<uint8_t>(hl[sb] >> 8);
            }
            if (lane == 0) reinterpret_cast<float *>(bt)[j] = d[sb];
            // 32-value bsum pairs: lane 4 i holds bsum 2 i, lane 4 i + 2 bsum 2 i + 1
            const int pair = bsv[sb] + __shfl_down_sync(0xffffffffu, bsv[sb], 2);
            if ((lane & 3) == 0)
                reinterpret_cast<int16_t *>(bt + MMQ_BT_BS2 + 16 * j)[lane >> 2] = static_cast<int16_t>(pair);
        }
    }
}

__global__ void __launch_bounds__(256) mmq_gather_q8K_kernel(const uint8_t *__restrict__ x8, int nsb, int k, int ntc,
                                                             const int32_t *__restrict__ entries,
                                                             const int4 *__restrict__ chunks,
                                                             const int32_t *__restrict__ n_chunks,
                                                             uint8_t *__restrict__ btiles) {
    const int lane = threadIdx.x & 31;
    const int n_items = *n_chunks * ntc;
    for (int wg = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wg < n_items; wg += (gridDim.x * blockDim.x) >> 5)
        mmq_gather_slot(x8, nsb, k, ntc, entries, chunks, btiles, wg, lane);
}


// B tiles of the 32-weight-block types, per chunk and step of sk values:
// the tokens' Q8_0 block scales (f16 -> float, [MMQ_NT32][8], blocks of the
// step), then the quants in the MMA's K-major layout (16-byte chunk c of
// token j at MMQ_BT32_HEAD + c * 16 N + (j / 8) * 128 + (j % 8) * 16). Copied
// from the tokens' Q8_0 rows x8 (34-byte blocks), one warp per token slot.
__global__ void __launch_bounds__(256) mmq_gather_q80_kernel(const uint8_t *__restrict__ x8, int K, int sk, int k,
                                                             int ntc, const int32_t *__restrict__ entries,
                                                             const int4 *__restrict__ chunks,
                                                             const int32_t *__restrict__ n_chunks,
                                                             uint8_t *__restrict__ btiles, uint32_t bt_stride) {
    const int lane = threadIdx.x & 31;
    const int nsb = K / sk, nb = sk / 32, per = sk / 32;   // bytes per lane and step: sk / 32
    const int n_items = *n_chunks * ntc;
    for (int wg = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wg < n_items; wg += (gridDim.x * blockDim.x) >> 5) {
        const int gc = wg / ntc, j = wg - gc * ntc;
        const int4 ch = chunks[gc];
        const int nt = ch.z, N = mmq_chunk_n(nt), CS = 16 * N;
        if (j >= N) continue;
        const int t = j < nt ? entries[ch.y + j] / k : -1;
        const uint8_t *row = x8 + static_cast<size_t>(t < 0 ? 0 : t) * (K / 32) * 34;
        for (int sb = 0; sb < nsb; ++sb) {
            uint8_t *bt = btiles + (static_cast<size_t>(gc) * nsb + sb) * bt_stride;
            const int e = lane * per, b = e / 32, o = e % 32;
            uint32_t w[2] = {0u, 0u};
            if (t >= 0) {
                const uint8_t *q = row + static_cast<size_t>(sb * nb + b) * 34 + 2 + o;
#pragma unroll
                for (int i = 0; i < 2; ++i)
                    if (4 * i < per)
                        w[i] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(q + 4 * i)) |
                               (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(q + 4 * i + 2)) << 16);
            }
            uint8_t *dst = bt + MMQ_BT32_HEAD + (e / 16) * CS + (j >> 3) * 128 + (j & 7) * 16 + (e % 16);
            if (per == 8) *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
            else *reinterpret_cast<uint32_t *>(dst) = w[0];
            if (lane < nb)
                reinterpret_cast<float *>(bt)[8 * j + lane] =
                    t >= 0 ? __half2float(*reinterpret_cast<const __half *>(row + static_cast<size_t>(sb * nb + lane) * 34))
                           : 0.f;
        }
    }
}

// The same B tiles quantized here from f32 rows, one row per entry (k = 1):
// row r = x[r], or with u set GLU(op, x[r], u[r]) (the down projection's
// input made from the gate and up outputs); llama.cpp's quantize_row_q8_K_ref
// and the same GLU as glu_kernel, so the bits equal quantize_act of the f32 h.
__global__ void __launch_bounds__(256) mmq_gather_rows_kernel(const float *__restrict__ x, const float *__restrict__ u,
                                                              int glu_op, float glu_limit, int K,
                                                              const int32_t *__restrict__ entries,
                                                              const int4 *__restrict__ chunks,
                                                              const int32_t *__restrict__ n_chunks, int ntc,
                                                              uint8_t *__restrict__ btiles) {
    const int lane = threadIdx.x & 31;
    const int nsb = K / 256;
    const int n_items = *n_chunks * ntc;
    for (int wg = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wg < n_items; wg += (gridDim.x * blockDim.x) >> 5) {
        const int gc = wg / ntc, j = wg - gc * ntc;
        const int4 ch = chunks[gc];
        const int nt = ch.z, N = mmq_chunk_n(nt), CS = 16 * N;
        if (j >= N) continue;
        const int row = j < nt ? entries[ch.y + j] : -1;
        for (int sb = 0; sb < nsb; ++sb) {
            uint8_t *bt = btiles + (static_cast<size_t>(gc) * nsb + sb) * MMQ_BT_BYTES;
            uint8_t *tok = bt + MMQ_BT_HEAD + (j >> 3) * 128 + (j & 7) * 16;
            int8_t q[8];
            int s = 0;
            float d = 0.f;
            if (row >= 0) {
                const float *xr = x + static_cast<size_t>(row) * K + sb * 256 + lane * 8;
                const float4 a0 = *reinterpret_cast<const float4 *>(xr), a1 = *reinterpret_cast<const float4 *>(xr + 4);
                float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                if (u) {
                    const float *ur = u + static_cast<size_t>(row) * K + sb * 256 + lane * 8;
                    const float4 b0 = *reinterpret_cast<const float4 *>(ur), b1 = *reinterpret_cast<const float4 *>(ur + 4);
                    const float w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = glu_apply(glu_op, v[i], w[i], glu_limit);
                }
                d = quant_q8K_vals(v, lane, q, s);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = 0;
            }
            uint32_t lo4 = 0, hi4 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo4 |= static_cast<uint32_t>(static_cast<uint8_t>(q[i])) << (8 * i);
                hi4 |= static_cast<uint32_t>(static_cast<uint8_t>(q[4 + i])) << (8 * i);
            }
            *reinterpret_cast<uint2 *>(tok + (lane >> 1) * CS + 8 * (lane & 1)) = make_uint2(lo4, hi4);
            if ((lane & 1) == 0) {
                tok[16 * CS + (lane >> 1)] = static_cast<uint8_t>((s >> 4) & 0xFF);
                tok[17 * CS + (lane >> 1)] = static_cast<uint8_t>(s & 15);
            }
            if (lane == 0) reinterpret_cast<float *>(bt)[j] = d;
            const int pair = s + __shfl_down_sync(0xffffffffu, s, 2);
            if ((lane & 3) == 0)
                reinterpret_cast<int16_t *>(bt + MMQ_BT_BS2 + 16 * j)[lane >> 2] = static_cast<int16_t>(pair);
        }
    }
}

// ---------------------------------------------------------------------------
// The grouped GEMM
// ---------------------------------------------------------------------------
// Per weight type: bytes per super-block, int8 planes of the folded weights
// (plane 0 = low byte, plane 1 = high byte of a 16-bit fold), whether plane p
// is signed, the mins term (Q2_K on the tensor core, Q4_K with dp2a in the
// epilogue) and the tokens per chunk (TMEM: two accumulator sets of
// (planes + summs) x NT columns plus two A buffers of 64 columns per plane:
// 512 columns at most).
//
// Q4_0, Q5_0 and Q8_0 (B32) carry one float scale per 32 weights and meet Q8_0
// activations (one scale per 32 values): a step is SK weights per row (256,
// or 128 for Q8_0's 34-byte blocks), each of its K = 32 MMAs goes to its own
// accumulator, and the epilogue applies llama.cpp's per-block float steps.
template <int TYPE>
struct MmqType;
template <> struct MmqType<T_Q2_K> {
    static constexpr int BPB = 84, NPLANE = 1, NT = 64, SK = 256, BLK = 0;
    static constexpr bool MINS_TC = true, MINS_DP = false, P0_SIGNED = false, P1_SIGNED = false, B32 = false;
};
template <> struct MmqType<T_Q3_K> {
    static constexpr int BPB = 110, NPLANE = 1, NT = 64, SK = 256, BLK = 0;
    static constexpr bool MINS_TC = false, MINS_DP = false, P0_SIGNED = true, P1_SIGNED = false, B32 = false;
};
template <> struct MmqType<T_Q4_K> {
    static constexpr int BPB = 144, NPLANE = 2, NT = 64, SK = 256, BLK = 0;
    static constexpr bool MINS_TC = false, MINS_DP = true, P0_SIGNED = false, P1_SIGNED = false, B32 = false;
};
template <> struct MmqType<T_Q5_K> {
    static constexpr int BPB = 176, NPLANE = 2, NT = 64, SK = 256, BLK = 0;
    static constexpr bool MINS_TC = false, MINS_DP = true, P0_SIGNED = false, P1_SIGNED = false, B32 = false;
};
template <> struct MmqType<T_Q6_K> {
    static constexpr int BPB = 210, NPLANE = 2, NT = 64, SK = 256, BLK = 0;
    static constexpr bool MINS_TC = false, MINS_DP = false, P0_SIGNED = false, P1_SIGNED = true, B32 = false;
};
template <> struct MmqType<T_Q4_0> {
    static constexpr int BLK = 18, SK = 256, BPB = BLK * SK / 32, NPLANE = 1, NT = MMQ_NT32;
    static constexpr bool MINS_TC = false, MINS_DP = false, P0_SIGNED = true, P1_SIGNED = false, B32 = true;
};
template <> struct MmqType<T_Q5_0> {
    static constexpr int BLK = 22, SK = 256, BPB = BLK * SK / 32, NPLANE = 1, NT = MMQ_NT32;
    static constexpr bool MINS_TC = false, MINS_DP = false, P0_SIGNED = true, P1_SIGNED = false, B32 = true;
};
template <> struct MmqType<T_Q8_0> {
    static constexpr int BLK = 34, SK = 128, BPB = BLK * SK / 32, NPLANE = 1, NT = MMQ_NT32;
    static constexpr bool MINS_TC = false, MINS_DP = false, P0_SIGNED = true, P1_SIGNED = false, B32 = true;
};

// Shared-memory and TMEM layout of one CTA for weight type TYPE. TMEM
// columns: accumulator set s at s * ACC_COLS (plane p at p * NT, summs after
// the planes), A buffer b at A_COL0 + b * A_COLS (plane p: 64 columns at
// p * 64, then the Q2_K mins: 8 columns).
template <int TYPE>
struct MmqLayout {
    using Ty = MmqType<TYPE>;
    static constexpr uint32_t SLOT = (Ty::BPB + 15) / 16 * 16 + 16;     // one row's window of one super-block
    static constexpr uint32_t CTRL = 16384;
    static constexpr int NB = 4;                                         // B-tile stages
    static constexpr uint32_t OFF_B = CTRL;
    static constexpr uint32_t OFF_P = (OFF_B + NB * MMQ_BT_BYTES + 127) / 128 * 128;
    static constexpr uint32_t STAGE = MMQ_M * SLOT;
    static constexpr int NP_FIT = static_cast<int>((227u * 1024u - OFF_P) / STAGE);
    static constexpr int NP = NP_FIT > 8 ? 8 : NP_FIT;                   // weight stages
    static constexpr uint32_t TOTAL = OFF_P + NP * STAGE;
    static constexpr uint32_t SUMMS_COL = Ty::NPLANE * Ty::NT;           // summs plane within a set
    // B32: one accumulator of NT columns per 32-weight block of the step
    static constexpr uint32_t ACC_COLS = Ty::B32 ? (Ty::SK / 32) * Ty::NT : SUMMS_COL + (Ty::MINS_TC ? Ty::NT : 0);
    static constexpr uint32_t A_COL0 = 2 * ACC_COLS;
    static constexpr uint32_t MINS_COL = Ty::NPLANE * 64;                // Q2_K mins within an A buffer
    static constexpr uint32_t A_COLS = Ty::B32 ? Ty::SK / 4 : MINS_COL + (Ty::MINS_TC ? 8 : 0);
    static_assert(NP >= 2, "at least two weight stages");
    static_assert(TOTAL <= 227u * 1024u, "shared memory budget");
    static_assert(A_COL0 + 2 * A_COLS <= 512, "TMEM columns");
    static_assert(SLOT % 16 == 0 && SLOT <= 256, "TMA box width");
    static_assert(Ty::NT == 32 || Ty::NT == 64 || (Ty::B32 && Ty::NT == MMQ_NT32), "chunk width");
};

// Warp roles: warps 0-7 finish the accumulators (warp w reads TMEM lanes
// 32 (w % 4) .. + 31, i.e. those weight rows, for the 16-token slices
// w / 4, w / 4 + 2), warps 8-15 unpack the weights (warp 8 + i: rows
// 32 (i % 4) + lane, elements 128 (i / 4) .. + 127 of each super-block),
// warp 16 loads, warps 17 and 18 issue the MMAs of the even and the odd steps
// (an MMA instruction holds its issuing thread for ~100 cycles whatever N; two
// issuers overlap).
constexpr int MMQ_EPI_WARPS = 8;
constexpr int MMQ_UNP_WARPS = 8;
constexpr int MMQ_PROD_WARP = MMQ_EPI_WARPS + MMQ_UNP_WARPS;
constexpr int MMQ_MMA_WARP = MMQ_PROD_WARP + 1;   // and MMQ_MMA_WARP + 1
constexpr int MMQ_WS_THREADS = 32 * (MMQ_MMA_WARP + 2);
constexpr int MMQ_RING = 4;   // steps of row and token scales kept for the epilogue

struct MmqCtrl {   // fits MmqLayout::CTRL (static_assert in the kernel)
    uint64_t p_full[8], p_empty[8], b_full[4], b_empty[4];
    uint64_t mma_done[2];      // step g's MMAs complete (accumulator set g & 1 full, A buffer g & 1 free)
    uint64_t acc_empty[2];     // the epilogue has read accumulator set g & 1
    uint64_t a_ready[2];       // step g's A buffer g & 1 unpacked
    uint64_t s_full[MMQ_RING]; // step g's row and token scales written
    uint32_t tmem;
    int32_t abort;             // a wait timed out somewhere: every role stops
    alignas(16) float da[MMQ_RING][MMQ_NT];
    union {
        alignas(16) int16_t bs2[MMQ_RING][MMQ_NT][8];        // Q4_K / Q5_K: the tokens' 32-value bsum pairs
        alignas(16) float da32[MMQ_RING][MMQ_NT32][8];       // B32: the tokens' block scales
    };
    union {
        struct {
            float2 rs[MMQ_RING][MMQ_M];                      // the rows' d, dmin
            uint2 rm[MMQ_RING][MMQ_M];                       // Q4_K / Q5_K: the rows' 8 mins (bytes)
        };
        __half rd[MMQ_RING][MMQ_M][8];                       // B32: the rows' block scales
    };
};

struct MmqTile {
    int e, rb, gchunk, first, nt;
};

// Tile ti = chunk ti / row_blocks, row block ti % row_blocks: consecutive
// tiles share the chunk and walk the row blocks.
__device__ __forceinline__ MmqTile mmq_tile(const int4 ch, int ti, int row_blocks) {
    MmqTile T;
    T.gchunk = ti / row_blocks;
    T.rb = ti - T.gchunk * row_blocks;
    T.e = ch.x;
    T.first = ch.y;
    T.nt = ch.z;
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

// ---- unpacking: half h (elements 128 h .. + 127) of one row's super-block
// into the A planes in TMEM (element k of plane p in byte k % 4 of column
// p * 64 + k / 4 of the thread's lane); half 0 also returns the row's scales.
// A word holds 4 consecutive elements; the 16-bit-lane helpers below fold a
// per-chunk scale into 4 elements at once: ev/od hold elements (0, 2) and
// (1, 3) in 16-bit lanes, sc * lanes + bias stays inside each lane.
struct RowScales {
    float d, dm;
    uint2 m;   // Q4_K mins
};

__device__ __forceinline__ uint32_t lo_bytes(uint32_t ev, uint32_t od) { return __byte_perm(ev, od, 0x6240); }
__device__ __forceinline__ uint32_t hi_bytes(uint32_t ev, uint32_t od) { return __byte_perm(ev, od, 0x7351); }
// 4 unsigned bytes x -> 16-bit lanes sc * x + bias (even and odd elements);
// b2 = bias * 0x10001
__device__ __forceinline__ void lane_fold(uint32_t x, int sc, int b2, uint32_t &ev, uint32_t &od) {
    ev = static_cast<uint32_t>(sc * static_cast<int>(__byte_perm(x, 0u, 0x4240)) + b2);   // bytes 0, 2
    od = static_cast<uint32_t>(sc * static_cast<int>(__byte_perm(x, 0u, 0x4341)) + b2);   // bytes 1, 3
}
// x >> s for s >= 0, x << -s otherwise
__device__ __forceinline__ uint32_t shr_signed(uint32_t x, int s) { return s >= 0 ? x >> s : x << -s; }

template <int TYPE>
__device__ __forceinline__ void mmq_unpack(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs);

// Q2_K (84 bytes: scales[16] (low nibble scale, high nibble min), qs[64],
// d, dmin): sc * q in [0, 45]; mins (16 m_g, m_g) for the summs MMA.
template <>
__device__ __forceinline__ void mmq_unpack<T_Q2_K>(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs) {
    uint32_t sc4[4], qs[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc4[i] = ld_u32(blk + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) qs[i] = ld_u32(blk + 16 + 32 * h + 4 * i);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t v[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            // elements 16 kb .. + 15 (kb = 8 h + c): plane c / 2 of quant bytes
            // 16 (c % 2) .. + 15 of the half's 32 bytes; one scale
            const int c = 4 * part + cc, kb = 8 * h + c, plane = c >> 1, hb = c & 1;
            const uint32_t sc = (sc4[kb >> 2] >> (8 * (kb & 3))) & 0xFu;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[4 * cc + i] = ((qs[4 * hb + i] >> (2 * plane)) & 0x03030303u) * sc;
        }
        tmem_st16(a_cols + 32 * h + 16 * part, v);
    }
    if (h == 0) {
        const uint32_t m[8] = {sc4[0] & 0xF0F0F0F0u, sc4[1] & 0xF0F0F0F0u, sc4[2] & 0xF0F0F0F0u, sc4[3] & 0xF0F0F0F0u,
                               (sc4[0] >> 4) & 0x0F0F0F0Fu, (sc4[1] >> 4) & 0x0F0F0F0Fu, (sc4[2] >> 4) & 0x0F0F0F0Fu,
                               (sc4[3] >> 4) & 0x0F0F0F0Fu};
        tmem_st8(a_cols + MmqLayout<T_Q2_K>::MINS_COL, m);
        rs.d = ld_half(blk + 80);
        rs.dm = ld_half(blk + 82);
    }
}

// Q3_K (110 bytes: hmask[32], qs[64], scales[12] (16 six-bit values, +32), d):
// value u - 4 with u = 2 low bits | high bit << 2; the plane holds
// -(sc - 32) * (u - 4) in [-128, 124], so isum = -(plane dot).
template <>
__device__ __forceinline__ void mmq_unpack<T_Q3_K>(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs) {
    uint32_t hm[8], qs[8], sw[3];
    ld_words_a2(blk, hm);
    ld_words_a2(blk + 32 + 32 * h, qs);
    ld_words_a2(blk + 96, sw);
    // the half's 8 scales (ggml's 6-bit scale unpacking, kmask1/kmask2)
    const uint32_t s_lo = h == 0 ? ((sw[0] & 0x0F0F0F0Fu) | (((sw[2] >> 0) & 0x03030303u) << 4))
                                 : (((sw[0] >> 4) & 0x0F0F0F0Fu) | (((sw[2] >> 4) & 0x03030303u) << 4));
    const uint32_t s_hi = h == 0 ? ((sw[1] & 0x0F0F0F0Fu) | (((sw[2] >> 2) & 0x03030303u) << 4))
                                 : (((sw[1] >> 4) & 0x0F0F0F0Fu) | (((sw[2] >> 6) & 0x03030303u) << 4));
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t v[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            // chunk c: shift j = c / 2, 16-element half c % 2 of the 32
            const int c = 4 * part + cc, j = c >> 1, hh = c & 1;
            const int s = static_cast<int>(((c < 4 ? s_lo : s_hi) >> (8 * (c & 3))) & 0xFFu) - 32;
            const int b2 = (4 * s + 256) * 0x10001;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // u = 2 low bits | high bit << 2 (the high bit moved straight to bit 2)
                const uint32_t u = ((qs[4 * hh + i] >> (2 * j)) & 0x03030303u) |
                                   (shr_signed(hm[4 * hh + i], 4 * h + j - 2) & 0x04040404u);
                uint32_t ev, od;
                lane_fold(u, -s, b2, ev, od);   // -s u + 4 s + 256 in [132, 384]
                v[4 * cc + i] = lo_bytes(ev, od);
            }
        }
        tmem_st16(a_cols + 32 * h + 16 * part, v);
    }
    if (h == 0) rs.d = ld_half(blk + 108);
}

// Q4_K (144 bytes: d, dmin, scales[12] (8 six-bit scales and mins), qs[128]):
// sc * q in [0, 945] as two planes (low byte, high byte).
__device__ __forceinline__ void q4K_scale_min(const uint32_t (&sw)[3], int j, int &sc, int &m) {
    const auto byte = [&](int i) { return static_cast<int>((sw[i >> 2] >> (8 * (i & 3))) & 0xFFu); };
    if (j < 4) {
        sc = byte(j) & 63;
        m = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

template <>
__device__ __forceinline__ void mmq_unpack<T_Q4_K>(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs) {
    uint32_t sw[3], qs[16];
#pragma unroll
    for (int i = 0; i < 3; ++i) sw[i] = ld_u32(blk + 4 + 4 * i);
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = ld_u32(blk + 16 + 64 * h + 4 * i);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            // chunk c: 32-byte group c / 4 of the half's 64 quant bytes, nibble
            // (c / 2) % 2, bytes 16 (c % 2) .. + 15; sub-block 4 h + 2 (c / 4) + (c / 2) % 2
            const int c = 4 * part + cc, nib = (c >> 1) & 1;
            int sc, m;
            q4K_scale_min(sw, 4 * h + 2 * (c >> 2) + nib, sc, m);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = qs[8 * (c >> 2) + 4 * (c & 1) + i] >> (4 * nib);
                const uint32_t ev = static_cast<uint32_t>(sc) * (w & 0x000F000Fu);          // elements 0, 2
                const uint32_t od = static_cast<uint32_t>(sc) * ((w >> 8) & 0x000F000Fu);   // elements 1, 3
                lo[4 * cc + i] = lo_bytes(ev, od);
                hi[4 * cc + i] = hi_bytes(ev, od);
            }
        }
        tmem_st16(a_cols + 32 * h + 16 * part, lo);
        tmem_st16(a_cols + 64 + 32 * h + 16 * part, hi);
    }
    if (h == 0) {
        uint32_t mb[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4K_scale_min(sw, j, sc, m);
            mb[j >> 2] |= static_cast<uint32_t>(m) << (8 * (j & 3));
        }
        rs.m = make_uint2(mb[0], mb[1]);
        rs.d = ld_half(blk);
        rs.dm = ld_half(blk + 2);
    }
}

// Q5_K (176 bytes: d, dmin, scales[12] (Q4_K's 6-bit scales and mins),
// qh[32], qs[128]): element l of 64-element group j is the nibble (j's 32
// bytes, low nibble for the group's first 32 elements, high for the rest)
// plus 16 * bit (2 j + half) of qh[l % 32]; sc * q in [0, 1953] as two
// unsigned planes; mins as Q4_K.
template <>
__device__ __forceinline__ void mmq_unpack<T_Q5_K>(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs) {
    uint32_t sw[3], qs[16], qh[8];
#pragma unroll
    for (int i = 0; i < 3; ++i) sw[i] = ld_u32(blk + 4 + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) qh[i] = ld_u32(blk + 16 + 4 * i);
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = ld_u32(blk + 48 + 64 * h + 4 * i);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            // chunk c as in Q4_K: group 2 h + c / 4, nibble (c / 2) % 2, bytes 16 (c % 2) .. + 15
            const int c = 4 * part + cc, nib = (c >> 1) & 1, grp = 2 * h + (c >> 2);
            int sc, m;
            q4K_scale_min(sw, 4 * h + 2 * (c >> 2) + nib, sc, m);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = (qs[8 * (c >> 2) + 4 * (c & 1) + i] >> (4 * nib)) & 0x0F0F0F0Fu;
                const uint32_t q = w | (((qh[4 * (c & 1) + i] >> (2 * grp + nib)) & 0x01010101u) << 4);
                const uint32_t ev = static_cast<uint32_t>(sc) * (q & 0x00FF00FFu);          // elements 0, 2
                const uint32_t od = static_cast<uint32_t>(sc) * ((q >> 8) & 0x00FF00FFu);   // elements 1, 3
                lo[4 * cc + i] = lo_bytes(ev, od);
                hi[4 * cc + i] = hi_bytes(ev, od);
            }
        }
        tmem_st16(a_cols + 32 * h + 16 * part, lo);
        tmem_st16(a_cols + 64 + 32 * h + 16 * part, hi);
    }
    if (h == 0) {
        uint32_t mb[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4K_scale_min(sw, j, sc, m);
            mb[j >> 2] |= static_cast<uint32_t>(m) << (8 * (j & 3));
        }
        rs.m = make_uint2(mb[0], mb[1]);
        rs.d = ld_half(blk);
        rs.dm = ld_half(blk + 2);
    }
}

// ---- the 32-weight-block types: half h of a step holds blocks
// [h NB / 2, (h + 1) NB / 2) of the row (NB = SK / 32), each 32 signed int8
// weights into 8 TMEM columns; the blocks' f16 scales go to rd[b]. Block
// starts are 2-byte aligned (18-, 22- and 34-byte blocks).
__device__ __forceinline__ uint32_t ld_u16x2(const uint8_t *p) {
    return static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(p)) |
           (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(p + 2)) << 16);
}

template <int TYPE>
__device__ __forceinline__ void mmq_unpack32(const uint8_t *step, uint32_t a_cols, int h, __half *rd) {
    using Ty = MmqType<TYPE>;
    constexpr int NB = Ty::SK / 32, BLK = Ty::BLK;
#pragma unroll
    for (int bb = 0; bb < NB / 2; ++bb) {
        const int b = h * (NB / 2) + bb;
        const uint8_t *blk = step + b * BLK;
        uint32_t v[8];
        if constexpr (TYPE == T_Q4_0) {
            // qs[16] at 2: element j = low nibble of qs[j] - 8, element 16 + j = high nibble - 8
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = ld_u16x2(blk + 2 + 4 * i);
                v[i] = __vsub4(w & 0x0F0F0F0Fu, 0x08080808u);
                v[4 + i] = __vsub4((w >> 4) & 0x0F0F0F0Fu, 0x08080808u);
            }
        } else if constexpr (TYPE == T_Q5_0) {
            // qh (32 bits) at 2, qs[16] at 6: the fifth bit of element j is qh bit j
            const uint32_t qh = ld_u16x2(blk + 2);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = ld_u16x2(blk + 6 + 4 * i);
                v[i] = __vsub4((w & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i)), 0x10101010u);
                v[4 + i] = __vsub4(((w >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i)), 0x10101010u);
            }
        } else {
            // Q8_0: qs[32] (int8) at 2
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = ld_u16x2(blk + 2 + 4 * i);
        }
        tmem_st8(a_cols + 8 * b, v);
        rd[b] = *reinterpret_cast<const __half *>(blk);
    }
}

// Q6_K (210 bytes: ql[128], qh[64], scales[16] (int8), d): sc * (q - 32) in
// [-4064, 4096] as two planes (low byte unsigned, high byte signed).
template <>
__device__ __forceinline__ void mmq_unpack<T_Q6_K>(const uint8_t *blk, uint32_t a_cols, int h, RowScales &rs) {
    uint32_t ql[16], qh[8], sw[2];
    ld_words_a2(blk + 64 * h, ql);
    ld_words_a2(blk + 128 + 32 * h, qh);
    ld_words_a2(blk + 192 + 8 * h, sw);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            // chunk c: group g = c / 2 (ql bytes 32 (g % 2) .., nibble g / 2,
            // qh bits 2 g), 16-element half c % 2 of the 32; scale 8 h + c
            const int c = 4 * part + cc, g = c >> 1, lh = c & 1;
            const int sc = static_cast<int>(static_cast<int8_t>((sw[c >> 2] >> (8 * (c & 3))) & 0xFFu));
            const int b2 = (32768 - 32 * sc) * 0x10001;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // q = low nibble | 2 high bits << 4 (moved straight to bits 4-5)
                const uint32_t q = ((ql[8 * (g & 1) + 4 * lh + i] >> (4 * (g >> 1))) & 0x0F0F0F0Fu) |
                                   (shr_signed(qh[4 * lh + i], 2 * g - 4) & 0x30303030u);
                uint32_t ev, od;
                lane_fold(q, sc, b2, ev, od);   // sc (q - 32) + 32768
                lo[4 * cc + i] = lo_bytes(ev, od);
                hi[4 * cc + i] = hi_bytes(ev, od) ^ 0x80808080u;
            }
        }
        tmem_st16(a_cols + 32 * h + 16 * part, lo);
        tmem_st16(a_cols + 64 + 32 * h + 16 * part, hi);
    }
    if (h == 0) rs.d = ld_half(blk + 208);
}

// Instruction descriptor of kind::i8 with s32 accumulation: A unsigned or
// signed int8, B signed int8, both K-major
__host__ __device__ constexpr uint32_t mmq_idesc(bool a_signed, int N) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(MMQ_M >> 4) << 24);
}

// summs of Q4_K: sum over the 8 sub-blocks of m_j * (bsum 2 j + bsum 2 j + 1)
__device__ __forceinline__ int q4K_summs(const int16_t *bs2, uint2 m) {
    const int4 b = *reinterpret_cast<const int4 *>(bs2);
    int acc = __dp2a_lo(b.x, static_cast<int>(m.x), 0);
    acc = __dp2a_hi(b.y, static_cast<int>(m.x), acc);
    acc = __dp2a_lo(b.z, static_cast<int>(m.y), acc);
    return __dp2a_hi(b.w, static_cast<int>(m.y), acc);
}

template <int TYPE>
__global__ void __launch_bounds__(MMQ_WS_THREADS, 1) moe_mmq_kernel(const __grid_constant__ MmqArgs a) {
    using Lay = MmqLayout<TYPE>;
    using Ty = MmqType<TYPE>;
    static_assert(sizeof(MmqCtrl) <= Lay::CTRL, "control block too large");
    constexpr int BPB = Ty::BPB, NT = Ty::NT;
    extern __shared__ __align__(1024) uint8_t smem[];
    MmqCtrl &C = *reinterpret_cast<MmqCtrl *>(smem);
    uint8_t *B = smem + Lay::OFF_B;
    uint8_t *P = smem + Lay::OFF_P;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nsb = a.K / Ty::SK;
    const int row_blocks = a.nrows / MMQ_M;
    const int total = *a.n_chunks * row_blocks;
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
        int4 ch = static_cast<int>(blockIdx.x) < total ? a.chunks[blockIdx.x / row_blocks] : make_int4(0, 0, 0, 0);
        for (int ti = blockIdx.x; ti < total && pok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(ch, ti, row_blocks);
            if (ti + static_cast<int>(gridDim.x) < total) ch = a.chunks[(ti + gridDim.x) / row_blocks];   // next tile's chunk
            const uint32_t bbytes = Ty::B32 ? mmq_bt32_bytes(mmq_chunk_n(T.nt), Ty::SK) : mmq_bt_bytes(mmq_chunk_n(T.nt));
            const int y0 = (T.e * a.nrows + T.rb * MMQ_M) / G;   // first tensor-map row of the tile
            for (int sb = 0; sb < nsb; ++sb) {
                bool w = lane == 0 ? mmq_wait(C, &C.b_empty[bs], bph ^ 1u, a) : true;
                if (!__shfl_sync(0xffffffffu, w, 0)) { pok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&C.b_full[bs], bbytes);
                    bulk_g2s(B + bs * MMQ_BT_BYTES, a.btiles + (static_cast<size_t>(T.gchunk) * nsb + sb) * a.bt_stride,
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
            int4 ch = static_cast<int>(blockIdx.x) < total ? a.chunks[blockIdx.x / row_blocks] : make_int4(0, 0, 0, 0);
            for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
                const MmqTile T = mmq_tile(ch, ti, row_blocks);
                if (ti + static_cast<int>(gridDim.x) < total) ch = a.chunks[(ti + gridDim.x) / row_blocks];
                const int N = mmq_chunk_n(T.nt);
                const uint32_t bcs = 16u * N;   // B: bytes of one 16-byte K chunk over the N tokens
                const uint32_t id0 = mmq_idesc(Ty::P0_SIGNED, N), id1 = mmq_idesc(Ty::P1_SIGNED, N);
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
                    const uint32_t b0 = smem_u32(B + bs * MMQ_BT_BYTES) + (Ty::B32 ? MMQ_BT32_HEAD : MMQ_BT_HEAD);
                    const uint32_t d0 = tmem + par * Lay::ACC_COLS;
                    if constexpr (Ty::B32) {
                        // one accumulator per 32-weight block (its own float scales)
#pragma unroll
                        for (int kk = 0; kk < Ty::SK / 32; ++kk)
                            umma_i8_ts(d0 + kk * NT, a0 + 8 * kk, umma_desc(b0 + kk * 2 * bcs, bcs, 128), id0, 0u);
                    } else {
#pragma unroll
                        for (int p = 0; p < Ty::NPLANE; ++p)
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk)
                                umma_i8_ts(d0 + p * NT, a0 + p * 64 + 8 * kk, umma_desc(b0 + kk * 2 * bcs, bcs, 128),
                                           p == 0 ? id0 : id1, kk > 0 ? 1u : 0u);
                    }
                    if (Ty::MINS_TC)   // summs = sum_g (16 m_g) hi_g + m_g lo_g
                        umma_i8_ts(d0 + Lay::SUMMS_COL, a0 + Lay::MINS_COL, umma_desc(b0 + 16 * bcs, bcs, 128),
                                   mmq_idesc(false, N), 0u);
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
        // this thread's TMEM lane (row r) in the A buffers
        const uint32_t a_lane = tmem + (static_cast<uint32_t>(32 * (uw & 3)) << 16) + Lay::A_COL0;
        uint32_t ps = 0, pph = 0, bs = 0, bph = 0, g = 0;
        bool ok = true;
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
            for (int sb = 0; sb < nsb; ++sb, ++g) {
                // weight stage landed; A buffer g & 1 last read by step g - 2's MMAs
                ok = mmq_wait(C, &C.p_full[ps], pph, a) &&
                     (g < 2 || mmq_wait(C, &C.mma_done[g & 1u], ((g - 2) >> 1) & 1u, a));
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint8_t *slot = P + ps * Lay::STAGE + slot_off + ((row_in_group + static_cast<uint32_t>(sb) * BPB) & 15u);
                if constexpr (Ty::B32) {
                    mmq_unpack32<TYPE>(slot, a_lane + (g & 1u) * Lay::A_COLS, h, C.rd[g % MMQ_RING][r]);
                } else {
                    RowScales rsc{};
                    mmq_unpack<TYPE>(slot, a_lane + (g & 1u) * Lay::A_COLS, h, rsc);
                    if (h == 0) {
                        C.rs[g % MMQ_RING][r] = make_float2(rsc.d, rsc.dm);
                        if (Ty::MINS_DP) C.rm[g % MMQ_RING][r] = rsc.m;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.p_empty[ps]);
                if (++ps == Lay::NP) { ps = 0; pph ^= 1u; }
                if (uw < (Ty::B32 ? 4 : 2)) {   // half 0 copies the token scales
                    ok = mmq_wait(C, &C.b_full[bs], bph, a);
                    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                    const uint8_t *Bst = B + bs * MMQ_BT_BYTES;
                    if constexpr (Ty::B32) {
                        // token n = r / 8, block r % 8 (blocks past the step are not read)
                        (&C.da32[g % MMQ_RING][0][0])[r] = reinterpret_cast<const float *>(Bst)[r];
                    } else {
                        C.da[g % MMQ_RING][r] = reinterpret_cast<const float *>(Bst)[r];
                        if (Ty::MINS_DP)
                            *reinterpret_cast<int4 *>(C.bs2[g % MMQ_RING][r]) =
                                *reinterpret_cast<const int4 *>(Bst + MMQ_BT_BS2 + 16 * r);
                    }
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
    } else if constexpr (Ty::B32) {
        // ---------------- epilogue warps, 32-weight blocks -------------------------
        // thread: row r, tokens 8 half .. + 7; per block llama.cpp's float steps
        // (Q4_0: sumi * dx * dy, Q5_0: (dx * dy) * sumi, Q8_0: sumi * (dx * dy)),
        // blocks in order
        constexpr int NB = Ty::SK / 32;
        const int r = 32 * (warp & 3) + lane, half = warp >> 2;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        uint32_t g = 0;
        bool ok = true;
        int4 ch = static_cast<int>(blockIdx.x) < total ? a.chunks[blockIdx.x / row_blocks] : make_int4(0, 0, 0, 0);
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(ch, ti, row_blocks);
            if (ti + static_cast<int>(gridDim.x) < total) ch = a.chunks[(ti + gridDim.x) / row_blocks];
            for (int sb = 0; sb < nsb; ++sb, ++g) {
                ok = mmq_wait(C, &C.s_full[g % MMQ_RING], (g / MMQ_RING) & 1u, a) &&
                     mmq_wait(C, &C.mma_done[g & 1u], (g >> 1) & 1u, a);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint32_t cols = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + (g & 1u) * Lay::ACC_COLS +
                                      8u * static_cast<uint32_t>(half);
                const __half *rdr = C.rd[g % MMQ_RING][r];
                const float *das = &C.da32[g % MMQ_RING][8 * half][0];
#pragma unroll
                for (int kk = 0; kk < NB; ++kk) {
                    uint32_t S[8];
                    tmem_ld8(cols + kk * NT, S);
                    tmem_wait_ld();
                    const float dx = __half2float(rdr[kk]);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float dy = das[8 * j + kk];
                        const float si = __int2float_rn(static_cast<int>(S[j]));
                        float t;
                        if constexpr (TYPE == T_Q4_0) t = __fmul_rn(__fmul_rn(si, dx), dy);
                        else if constexpr (TYPE == T_Q5_0) t = __fmul_rn(__fmul_rn(dx, dy), si);
                        else t = __fmul_rn(si, __fmul_rn(dx, dy));
                        acc[j] = __fadd_rn(acc[j], t);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.acc_empty[g & 1u]);
                if (sb == nsb - 1) {
                    const int row = T.rb * MMQ_M + r;
                    const int32_t *ent = a.entries + T.first;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int n = 8 * half + j;
                        if (n < T.nt) a.dst[static_cast<int64_t>(ent[n]) * a.nrows + row] = acc[j];
                        acc[j] = 0.f;
                    }
                }
            }
        }
    } else {
        // ---------------- epilogue warps -----------------------------------------
        constexpr int NQ = NT / 32;                               // 16-token slices per warp
        const int r = 32 * (warp & 3) + lane, half = warp >> 2;   // row; slices half + 2 q
        float acc[16 * NQ];
#pragma unroll
        for (int n = 0; n < 16 * NQ; ++n) acc[n] = 0.f;
        uint32_t g = 0;
        bool ok = true;
        int4 ch = static_cast<int>(blockIdx.x) < total ? a.chunks[blockIdx.x / row_blocks] : make_int4(0, 0, 0, 0);
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(ch, ti, row_blocks);
            if (ti + static_cast<int>(gridDim.x) < total) ch = a.chunks[(ti + gridDim.x) / row_blocks];
            for (int sb = 0; sb < nsb; ++sb, ++g) {
                ok = mmq_wait(C, &C.s_full[g % MMQ_RING], (g / MMQ_RING) & 1u, a) &&
                     mmq_wait(C, &C.mma_done[g & 1u], (g >> 1) & 1u, a);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint32_t cols = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + (g & 1u) * Lay::ACC_COLS;
                const float2 rs = C.rs[g % MMQ_RING][r];
                const float *dav = C.da[g % MMQ_RING];
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    const int sl = half + 2 * q;
                    if (sl * 16 < T.nt) {
                        uint32_t S0[16], S1[16];
                        tmem_ld16(cols + sl * 16, S0);
                        if (Ty::NPLANE == 2) tmem_ld16(cols + NT + sl * 16, S1);
                        if (Ty::MINS_TC) tmem_ld16(cols + Lay::SUMMS_COL + sl * 16, S1);
                        tmem_wait_ld();
                        float dv[16];
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 t4 = *reinterpret_cast<const float4 *>(dav + sl * 16 + j);
                            dv[j] = t4.x; dv[j + 1] = t4.y; dv[j + 2] = t4.z; dv[j + 3] = t4.w;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            float &A = acc[q * 16 + j];
                            const float dall = __fmul_rn(dv[j], rs.x);
                            if (TYPE == T_Q2_K) {
                                // llama.cpp's sumf += (d_a d) * isum - (d_a dmin) * summs
                                const float dmin = __fmul_rn(dv[j], rs.y);
                                const float fi = small_int_to_float(static_cast<int>(S0[j]));
                                const float fm = small_int_to_float(static_cast<int>(S1[j]));
                                A = __fadd_rn(A, __fsub_rn(__fmul_rn(dall, fi), __fmul_rn(dmin, fm)));
                            } else if (TYPE == T_Q3_K) {
                                A = __fadd_rn(A, __fmul_rn(dall, small_int_to_float(-static_cast<int>(S0[j]))));
                            } else {
                                const int isum = static_cast<int>(S0[j]) + 256 * static_cast<int>(S1[j]);
                                float t = __fmul_rn(dall, __int2float_rn(isum));
                                if (Ty::MINS_DP) {
                                    // - (d_a dmin) * summs
                                    const int sm = q4K_summs(C.bs2[g % MMQ_RING][sl * 16 + j], C.rm[g % MMQ_RING][r]);
                                    t = __fsub_rn(t, __fmul_rn(__fmul_rn(dv[j], rs.y), small_int_to_float(sm)));
                                }
                                A = __fadd_rn(A, t);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.acc_empty[g & 1u]);
                if (sb == nsb - 1) {
                    const int row = T.rb * MMQ_M + r;
                    const int32_t *ent = a.entries + T.first;
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
}

cudaError_t launch_mmq_group(const int32_t *ids, int64_t ids_stride, int n_tok, int k, int E, int ntc,
                             int32_t *entries, int4 *chunks, int32_t *n_chunks, int *err, cudaStream_t st,
                             bool skip_empty) {
    const size_t smem = static_cast<size_t>(E) * sizeof(int32_t);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(mmq_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    mmq_group_kernel<<<1, 1024, smem, st>>>(ids, ids_stride, n_tok, k, E, ntc, skip_empty ? 1 : 0, entries, chunks,
                                            n_chunks, err);
    return cudaGetLastError();
}

cudaError_t launch_mmq_gather(const uint8_t *x8, int K, int k, int ntc, const int32_t *entries, const int4 *chunks,
                              const int32_t *n_chunks, int64_t max_chunks, uint8_t *btiles, cudaStream_t st) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (max_chunks * ntc + 7) / 8;   // one warp per token slot, 8 warps a block
    const int grid = static_cast<int>(blocks < 8 * n_sm ? (blocks > 0 ? blocks : 1) : 8 * n_sm);
    mmq_gather_q8K_kernel<<<grid, 256, 0, st>>>(x8, K / 256, k, ntc, entries, chunks, n_chunks, btiles);
    return cudaGetLastError();
}

cudaError_t launch_mmq_gather32(const uint8_t *x8, int K, int sk, int k, int ntc, const int32_t *entries,
                                const int4 *chunks, const int32_t *n_chunks, int64_t max_chunks, uint8_t *btiles,
                                uint32_t bt_stride, cudaStream_t st) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (max_chunks * ntc + 7) / 8;   // one warp per token slot, 8 warps a block
    const int grid = static_cast<int>(blocks < 8 * n_sm ? (blocks > 0 ? blocks : 1) : 8 * n_sm);
    mmq_gather_q80_kernel<<<grid, 256, 0, st>>>(x8, K, sk, k, ntc, entries, chunks, n_chunks, btiles, bt_stride);
    return cudaGetLastError();
}

cudaError_t launch_mmq_gather_rows(const float *x, const float *u, int glu_op, float glu_limit, int K,
                                   const int32_t *entries, const int4 *chunks, const int32_t *n_chunks, int ntc,
                                   int64_t max_chunks, uint8_t *btiles, cudaStream_t st) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (max_chunks * ntc + 7) / 8;   // one warp per token slot, 8 warps a block
    const int grid = static_cast<int>(blocks < 8 * n_sm ? (blocks > 0 ? blocks : 1) : 8 * n_sm);
    mmq_gather_rows_kernel<<<grid, 256, 0, st>>>(x, u, glu_op, glu_limit, K, entries, chunks, n_chunks, ntc, btiles);
    return cudaGetLastError();
}

// Picks of a host-tiered tensor as pool slots: out[t * k + p] = the slot of
// expert ids[t][p] when its table entry points into the pool, else -1 (host
// memory: left to the GEMV). Out-of-range ids are left as they are (the
// grouping reports them).
__global__ void mmq_pool_ids_kernel(const int32_t *__restrict__ ids, int64_t ids_stride, int n_tok, int k,
                                    char *const *__restrict__ tbl, int n_experts, const char *pool,
                                    uint64_t expert_bytes, int n_slots, int32_t *out) {
    const int n = n_tok * k;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(pool);
    const uintptr_t hi = lo + static_cast<uintptr_t>(n_slots) * expert_bytes;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int t = i / k, p = i - t * k;
        const int x = ids[static_cast<int64_t>(t) * ids_stride + p];
        int v = x;
        if (x >= 0 && x < n_experts) {
            const uintptr_t q = reinterpret_cast<uintptr_t>(tbl[x]);
            v = (!(q & 1u) && q >= lo && q < hi) ? static_cast<int>((q - lo) / expert_bytes) : -1;
        } else if (x == -1) {
            v = n_slots;   // not a host pick either: out of range for the slot grouping (reported there)
        }
        out[i] = v;
    }
}

cudaError_t launch_mmq_pool_ids(const int32_t *ids, int64_t ids_stride, int n_tok, int k, char *const *tbl,
                                int n_experts, const char *pool, uint64_t expert_bytes, int n_slots, int32_t *out,
                                cudaStream_t st) {
    const int n = n_tok * k;
    const int grid = (n + 255) / 256 < 1024 ? ((n + 255) / 256 > 0 ? (n + 255) / 256 : 1) : 1024;
    mmq_pool_ids_kernel<<<grid, 256, 0, st>>>(ids, ids_stride, n_tok, k, tbl, n_experts, pool, expert_bytes, n_slots,
                                              out);
    return cudaGetLastError();
}

// The chunk table of a one-expert call whose ids are all 0 (the shared
// expert): entries in order, chunks of ntc consecutive entries.
__global__ void mmq_identity_chunks_kernel(int n, int ntc, int32_t *entries, int4 *chunks, int32_t *n_chunks) {
    const int nch = (n + ntc - 1) / ntc;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        entries[i] = i;
        if (i % ntc == 0) chunks[i / ntc] = make_int4(0, i, min(ntc, n - i), i / ntc);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_chunks = nch;
}

cudaError_t launch_mmq_identity_chunks(int n, int ntc, int32_t *entries, int4 *chunks, int32_t *n_chunks,
                                       cudaStream_t st) {
    const int grid = (n + 255) / 256 < 148 ? (n + 255) / 256 : 148;
    mmq_identity_chunks_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(n, ntc, entries, chunks, n_chunks);
    return cudaGetLastError();
}

int mmq_chunk_tokens(int type) {
    switch (type) {
        case T_Q2_K: return MmqType<T_Q2_K>::NT;
        case T_Q3_K: return MmqType<T_Q3_K>::NT;
        case T_Q4_K: return MmqType<T_Q4_K>::NT;
        case T_Q5_K: return MmqType<T_Q5_K>::NT;
        case T_Q6_K: return MmqType<T_Q6_K>::NT;
        case T_Q4_0: return MmqType<T_Q4_0>::NT;
        case T_Q5_0: return MmqType<T_Q5_0>::NT;
        case T_Q8_0: return MmqType<T_Q8_0>::NT;
        default: return 0;
    }
}

bool mmq_b32(int type) { return type == T_Q4_0 || type == T_Q5_0 || type == T_Q8_0; }

int mmq_step(int type) { return type == T_Q8_0 ? MmqType<T_Q8_0>::SK : 256; }

uint32_t mmq_bt_stride(int type) {
    return mmq_b32(type) ? (mmq_bt32_bytes(MMQ_NT32, mmq_step(type)) + 15u) / 16u * 16u : MMQ_BT_BYTES;
}

bool mmq_supported(int type, int64_t K, int64_t nrows) {
    if (mmq_chunk_tokens(type) <= 0 || nrows % MMQ_M != 0) return false;
    if (mmq_b32(type)) return K % mmq_step(type) == 0 && K <= 8192;
    return K % 256 == 0 && K / 256 <= MMQ_GATHER_MAX_SB;
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

template <int TYPE>
int launch_mmq_t(MmqArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    using Lay = MmqLayout<TYPE>;
    if ((reinterpret_cast<uintptr_t>(a.dense) & 15u) != 0 || !encode_rows_map(a, Lay::SLOT)) {
        *why = "cannot describe the expert rows as a TMA tensor map";
        return -2;
    }
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -3;
    auto kern = moe_mmq_kernel<TYPE>;
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

}  // namespace

int launch_mmq(int type, MmqArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    if (!mmq_supported(type, a.K, a.nrows)) {
        *why = "tensor-core prefill needs Q2_K..Q6_K (K % 256 == 0, K <= 4096) or Q4_0/Q5_0/Q8_0 (K <= 8192), "
               "rows % 128 == 0";
        return -2;
    }
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;
    if (a.bt_stride == 0) a.bt_stride = mmq_bt_stride(type);
    switch (type) {
        case T_Q4_0: return launch_mmq_t<T_Q4_0>(a, st, why, cuda_err);
        case T_Q5_0: return launch_mmq_t<T_Q5_0>(a, st, why, cuda_err);
        case T_Q8_0: return launch_mmq_t<T_Q8_0>(a, st, why, cuda_err);
        case T_Q2_K: return launch_mmq_t<T_Q2_K>(a, st, why, cuda_err);
        case T_Q3_K: return launch_mmq_t<T_Q3_K>(a, st, why, cuda_err);
        case T_Q4_K: return launch_mmq_t<T_Q4_K>(a, st, why, cuda_err);
        case T_Q5_K: return launch_mmq_t<T_Q5_K>(a, st, why, cuda_err);
        default: return launch_mmq_t<T_Q6_K>(a, st, why, cuda_err);
    }
}

}  // namespace moe
