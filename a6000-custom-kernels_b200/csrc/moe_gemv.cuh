// moe_gemv.cuh -- pointer-table quantized MUL_MAT_ID GEMV for sm_100a.
//
// Replaces the reference's moe_cache_gemv (kernels/moe-cache.cu:72-291) and its
// launch plumbing (:781-868). Same contract -- per (pick, token) one output row
// vector computed from the expert the pick routes to, read through a per-tensor
// pointer table whose LSB tags host-resident experts -- with a B200 structure:
//
//  * one CTA per SM; routed experts are de-duplicated inside the CTA, so each
//    expert's weights stream from HBM once per launch however many tokens
//    picked it (the reference re-reads them per (pick, token));
//  * the concatenated row space of all routed experts (+ the shared expert) is
//    split evenly over the CTAs;
//  * a producer warp streams contiguous row tiles into a shared-memory ring
//    with 1-D bulk copies (cp.async.bulk, mbarrier completion, no multicast);
//    host-tagged experts are copied by the same warp with plain loads;
//  * eight consumer warps dequantize in registers and run dp4a/dp2a integer
//    dots against activations staged once per CTA in shared memory, reduce
//    with warp shuffles and apply the fused bias / GLU / shared-expert
//    epilogue of the reference (:241-284);
//  * the first CTA does the reference's per-(pick, token) bookkeeping: stamps,
//    hit count and miss log (:163-198).
#pragma once
#include "moe_common.cuh"

namespace moe {

constexpr int GEMV_CONSUMER_WARPS = 8;
constexpr int GEMV_THREADS = 32 * (GEMV_CONSUMER_WARPS + 1);
constexpr int GEMV_MAX_ENTRIES = 256;    // ncols_dst * nchannels_dst
constexpr int GEMV_MAX_SEGMENTS = 32;
constexpr int GEMV_MAX_STAGES = 32;
constexpr int GEMV_MAX_KEYS = 272;
constexpr int GEMV_LOG_BASE = 2;         // stats: [0] misses, [1] hits, [2..] miss log
constexpr uint32_t KEY_SHARED = 0xFFFFu;

struct GemvArgs {
    // weights
    const char *const *tbl;        // [n_experts] tagged pointers of the main (up / down) tensor
    const char *const *tbl_gate;   // gate table, or null
    const char *gate_dense;        // gate base when it has no table (expert stride below)
    uint64_t gate_expert_bytes;
    const char *shared_up, *shared_gate;
    float *shared_dst;
    int64_t shared_stride_col_dst;
    const void *shared_y;          // activations of the shared block (null: channel 0 of y)
    int64_t shared_y_stride_col;
    // bookkeeping (reference :163-198)
    uint32_t *stamps, *stamps_gate;
    uint32_t *stats;
    const uint32_t *clock;
    int32_t cache_id, cache_id_gate;
    uint32_t log_cap;
    // activations: Q8_1 blocks (strides in blocks) or f32 (strides in floats)
    const void *y;
    int64_t stride_col_y, stride_channel_y;
    int32_t nchannels_y;
    // routing
    const int32_t *ids;
    int64_t ids_stride;
    int32_t ncols_dst, nchannels_dst, n_experts;
    // output
    float *dst;
    int64_t stride_col_dst, stride_channel_dst;
    // fusion (reference :109-129)
    int32_t has_fusion, use_gate;
    const float *x_bias, *gate_bias;
    int32_t glu_op;
    float glu_limit;
    // shape
    int32_t K, nrows;
    uint32_t row_bytes;
    // geometry (set by the launcher)
    int32_t lanes_per_row, rows_per_tile, n_stages, n_parts, act_slots;
    uint32_t part_bytes, slot_bytes, ctrl_bytes;
    int32_t tma_main, tma_gate, tma_shared;
    int *err;
    uint64_t timeout_ns;
};

// ---------------------------------------------------------------------------
// activations staged in shared memory, one slot per distinct input vector:
//   int8 q[K] | int16 bsum16[K/16] | f32 scale[K/32]
// scale is per 32 (Q8_0 / Q8_1) or per 256 (Q8_K, first K/256 entries).
// ---------------------------------------------------------------------------
template <int NMX>
struct Acts {
    const int8_t *q[NMX];
    const int16_t *bs[NMX];
    const float *sc[NMX];
    int nm;
};

__device__ __forceinline__ int bs_lo(int w) { return static_cast<int16_t>(w & 0xFFFF); }
__device__ __forceinline__ int bs_hi(int w) { return w >> 16; }

// Q8_K block (256) from f32: llama.cpp quantize_row_q8_K_ref, bit-exact.
__device__ __forceinline__ void stage_q8K_block(const float *x, int8_t *q, int16_t *bs, float *sc, int b, int lane) {
    float v[8];
    float amax = 0.f, mval = 0.f;
    int midx = 1 << 30;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = x[b * 256 + lane * 8 + j];
        const float ax = fabsf(v[j]);
        if (ax > amax) { amax = ax; mval = v[j]; midx = lane * 8 + j; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float ov = __shfl_xor_sync(0xffffffffu, mval, off);
        const int oi = __shfl_xor_sync(0xffffffffu, midx, off);
        if (oa > amax || (oa == amax && oi < midx)) { amax = oa; mval = ov; midx = oi; }
    }
    int8_t qq[8];
    float d = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int j = 0; j < 8; ++j) qq[j] = 0;
    } else {
        const float iscale = -127.f / mval;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = nearest_int_dev(__fmul_rn(iscale, v[j]));
            qq[j] = static_cast<int8_t>(r < 127 ? r : 127);
        }
        d = 1.f / iscale;
    }
    uint32_t w0 = 0, w1 = 0;
    int s = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        w0 |= (static_cast<uint32_t>(static_cast<uint8_t>(qq[j])) << (8 * j));
        w1 |= (static_cast<uint32_t>(static_cast<uint8_t>(qq[j + 4])) << (8 * j));
        s += qq[j] + qq[j + 4];
    }
    reinterpret_cast<uint2 *>(q + b * 256)[lane] = make_uint2(w0, w1);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) bs[b * 16 + (lane >> 1)] = static_cast<int16_t>(s);
    if (lane == 0) sc[b] = d;
}

// Q8_0 block (32) from f32: llama.cpp quantize_row_q8_0_ref, bit-exact.
__device__ __forceinline__ void stage_q80_block(const float *x, int8_t *q, int16_t *bs, float *sc, int b, int lane) {
    const float v = x[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = amax / 127.f;
    const float id = d != 0.f ? 1.0f / d : 0.0f;
    const int qi = static_cast<int>(roundf(__fmul_rn(v, id)));
    q[b * 32 + lane] = static_cast<int8_t>(qi);
    int s = qi;
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((lane & 15) == 0) bs[b * 2 + (lane >> 4)] = static_cast<int16_t>(s);
    if (lane == 0) sc[b] = __half2float(__float2half_rn(d));
}

// Q8_1 block (36 bytes) as given: copy qs, scale = d, per-16 sums.
__device__ __forceinline__ void stage_q81_block(const uint8_t *yb, int8_t *q, int16_t *bs, float *sc, int b, int lane) {
    const uint8_t *blk = yb + static_cast<size_t>(b) * 36;
    int s = 0;
    if (lane < 8) {
        const uint32_t w = ld_u32(blk + 4 + 4 * lane);
        reinterpret_cast<uint32_t *>(q + b * 32)[lane] = w;
        s = dp4a_ss(static_cast<int>(w), 0x01010101, 0);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (lane == 0) bs[b * 2] = static_cast<int16_t>(s);
    if (lane == 4) bs[b * 2 + 1] = static_cast<int16_t>(s);
    if (lane == 0) sc[b] = ld_half(blk);
}

// ---------------------------------------------------------------------------
// per-type task dots. A task is a fixed slice of one weight row; the lane adds
// its contribution for every member activation vector into acc[m].
// ---------------------------------------------------------------------------

// Q4_0 / Q5_0 / Q8_0: task = one 32-element block
template <int TYPE, int NMX>
__device__ __forceinline__ void task_legacy(const uint8_t *row, int b, const Acts<NMX> &A, float (&acc)[NMX]) {
    const uint8_t *blk = row + b * fmt<TYPE>::bytes;
    const float dw = ld_half(blk);
    uint32_t lo[4], hi[4];
    uint32_t w8[8];
    if constexpr (TYPE == T_Q4_0) {
        uint32_t w[4];
        ld_words_a2<4>(blk + 2, w);
#pragma unroll
        for (int i = 0; i < 4; ++i) { lo[i] = w[i] & 0x0F0F0F0Fu; hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu; }
    } else if constexpr (TYPE == T_Q5_0) {
        uint32_t w[5];
        ld_words_a2<5>(blk + 2, w);
        const uint32_t qh = w[0];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (w[1 + i] & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i));
            hi[i] = ((w[1 + i] >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i));
        }
    } else {
        ld_words_a2<8>(blk + 2, w8);
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = reinterpret_cast<const int4 *>(A.q[m] + b * 32);
        const int4 a0 = aq[0], a1 = aq[1];
        int S;
        if constexpr (TYPE == T_Q8_0) {
            S = dp4a_ss(static_cast<int>(w8[0]), a0.x, 0);
            S = dp4a_ss(static_cast<int>(w8[1]), a0.y, S);
            S = dp4a_ss(static_cast<int>(w8[2]), a0.z, S);
            S = dp4a_ss(static_cast<int>(w8[3]), a0.w, S);
            S = dp4a_ss(static_cast<int>(w8[4]), a1.x, S);
            S = dp4a_ss(static_cast<int>(w8[5]), a1.y, S);
            S = dp4a_ss(static_cast<int>(w8[6]), a1.z, S);
            S = dp4a_ss(static_cast<int>(w8[7]), a1.w, S);
        } else {
            S = dp4a_us(lo[0], a0.x, 0);
            S = dp4a_us(lo[1], a0.y, S);
            S = dp4a_us(lo[2], a0.z, S);
            S = dp4a_us(lo[3], a0.w, S);
            S = dp4a_us(hi[0], a1.x, S);
            S = dp4a_us(hi[1], a1.y, S);
            S = dp4a_us(hi[2], a1.z, S);
            S = dp4a_us(hi[3], a1.w, S);
            const int bsw = *reinterpret_cast<const int *>(A.bs[m] + b * 2);
            const int asum = bs_lo(bsw) + bs_hi(bsw);
            S -= (TYPE == T_Q4_0 ? 8 : 16) * asum;
        }
        acc[m] += (dw * A.sc[m][b]) * static_cast<float>(S);
    }
}

// Q2_K: task = (super-block, 128-element half n)
template <int ACT, int NMX>
__device__ __forceinline__ void task_q2_K(const uint8_t *row, int t, const Acts<NMX> &A, float (&acc)[NMX]) {
    const int sb = t >> 1, n = t & 1;
    const uint8_t *blk = row + sb * 84;
    uint32_t q[8];
    ld_words_a4<8>(blk + 16 + 32 * n, q);
    const uint32_t sw0 = ld_u32(blk + 8 * n), sw1 = ld_u32(blk + 8 * n + 4);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(blk + 80));
    const uint32_t mw0 = (sw0 >> 4) & 0x0F0F0F0Fu, mw1 = (sw1 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = reinterpret_cast<const int4 *>(A.q[m] + sb * 256 + 128 * n);
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + sb * 16 + 8 * n);
        int Ih = 0;
        float fI = 0.f, fM = 0.f;
#pragma unroll
        for (int k = 3; k >= 0; --k) {
            const uint32_t M = 0x03030303u << (2 * k);
            const int4 a0 = aq[2 * k], a1 = aq[2 * k + 1];
            int S0 = dp4a_us(q[0] & M, a0.x, 0);
            S0 = dp4a_us(q[1] & M, a0.y, S0);
            S0 = dp4a_us(q[2] & M, a0.z, S0);
            S0 = dp4a_us(q[3] & M, a0.w, S0);
            int S1 = dp4a_us(q[4] & M, a1.x, 0);
            S1 = dp4a_us(q[5] & M, a1.y, S1);
            S1 = dp4a_us(q[6] & M, a1.z, S1);
            S1 = dp4a_us(q[7] & M, a1.w, S1);
            const uint32_t sw = k < 2 ? sw0 : sw1;
            const int sc0 = (sw >> (16 * (k & 1))) & 0xF;
            const int sc1 = (sw >> (16 * (k & 1) + 8)) & 0xF;
            const int Ik = sc0 * S0 + sc1 * S1;   // 4^k times the true value (exact)
            if constexpr (ACT == ACT_CPU) {
                Ih = (k == 3) ? Ik : (Ih >> 2) + Ik;
            } else {
                const float d8 = A.sc[m][sb * 8 + 4 * n + k];
                const int bw = k == 0 ? bsv.x : k == 1 ? bsv.y : k == 2 ? bsv.z : bsv.w;
                const uint32_t mw = k < 2 ? mw0 : mw1;
                const int Mk = (k & 1) ? dp2a_hi_su(bw, mw, 0) : dp2a_lo_su(bw, mw, 0);
                fI += d8 * static_cast<float>(Ik >> (2 * k));
                fM += d8 * static_cast<float>(Mk);
            }
        }
        if constexpr (ACT == ACT_CPU) {
            int Mi = dp2a_lo_su(bsv.x, mw0, 0);
            Mi = dp2a_hi_su(bsv.y, mw0, Mi);
            Mi = dp2a_lo_su(bsv.z, mw1, Mi);
            Mi = dp2a_hi_su(bsv.w, mw1, Mi);
            const float d8 = A.sc[m][sb];
            acc[m] += d8 * (dm.x * static_cast<float>(Ih) - dm.y * static_cast<float>(Mi));
        } else {
            acc[m] += dm.x * fI - dm.y * fM;
        }
    }
}

// Q3_K: task = (super-block, 128-element half n)
template <int ACT, int NMX>
__device__ __forceinline__ void task_q3_K(const uint8_t *row, int t, const Acts<NMX> &A, float (&acc)[NMX]) {
    const int sb = t >> 1, n = t & 1;
    const uint8_t *blk = row + sb * 110;
    uint32_t qw[8], hw[8], sc3[3];
    ld_words_a2<8>(blk + 32 + 32 * n, qw);
    ld_words_a2<8>(blk, hw);
    ld_words_a2<3>(blk + 96, sc3);
    const float d = ld_half(blk + 108);
    uint32_t SW0, SW1;   // scale + 32 for sub-blocks 8n + 0..3 and 8n + 4..7
    if (n == 0) {
        SW0 = (sc3[0] & 0x0F0F0F0Fu) | ((sc3[2] & 0x03030303u) << 4);
        SW1 = (sc3[1] & 0x0F0F0F0Fu) | (((sc3[2] >> 2) & 0x03030303u) << 4);
    } else {
        SW0 = ((sc3[0] >> 4) & 0x0F0F0F0Fu) | (((sc3[2] >> 4) & 0x03030303u) << 4);
        SW1 = ((sc3[1] >> 4) & 0x0F0F0F0Fu) | (((sc3[2] >> 6) & 0x03030303u) << 4);
    }
    uint32_t u[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int hs = 4 * n + k;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            u[k][i] = ((qw[i] >> (2 * k)) & 0x03030303u) | (((hw[i] >> hs) & 0x01010101u) << 2);
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = reinterpret_cast<const int4 *>(A.q[m] + sb * 256 + 128 * n);
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + sb * 16 + 8 * n);
        const int bsw[4] = {bsv.x, bsv.y, bsv.z, bsv.w};
        int I = 0;
        float fI = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int4 a0 = aq[2 * k], a1 = aq[2 * k + 1];
            int S0 = dp4a_us(u[k][0], a0.x, 0);
            S0 = dp4a_us(u[k][1], a0.y, S0);
            S0 = dp4a_us(u[k][2], a0.z, S0);
            S0 = dp4a_us(u[k][3], a0.w, S0);
            int S1 = dp4a_us(u[k][4], a1.x, 0);
            S1 = dp4a_us(u[k][5], a1.y, S1);
            S1 = dp4a_us(u[k][6], a1.z, S1);
            S1 = dp4a_us(u[k][7], a1.w, S1);
            const uint32_t SW = k < 2 ? SW0 : SW1;
            const int s0 = static_cast<int>((SW >> (16 * (k & 1))) & 0xFF) - 32;
            const int s1 = static_cast<int>((SW >> (16 * (k & 1) + 8)) & 0xFF) - 32;
            const int Ik = s0 * (S0 - 4 * bs_lo(bsw[k])) + s1 * (S1 - 4 * bs_hi(bsw[k]));
            if constexpr (ACT == ACT_CPU) I += Ik;
            else fI += A.sc[m][sb * 8 + 4 * n + k] * static_cast<float>(Ik);
        }
        if constexpr (ACT == ACT_CPU) acc[m] += A.sc[m][sb] * (d * static_cast<float>(I));
        else acc[m] += d * fI;
    }
}

// Q4_K / Q5_K: task = (super-block, 64-element chunk c) = sub-blocks 2c, 2c+1
template <int TYPE, int ACT, int NMX>
__device__ __forceinline__ void task_q45_K(const uint8_t *row, int t, const Acts<NMX> &A, float (&acc)[NMX]) {
    const int sb = t >> 2, c = t & 3;
    const uint8_t *blk = row + sb * fmt<TYPE>::bytes;
    uint32_t qw[8];
    ld_words_a4<8>(blk + (TYPE == T_Q4_K ? 16 : 48) + 32 * c, qw);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(blk));
    const uint32_t Sw = ld_u32(blk + 4), Mw = ld_u32(blk + 8), Xw = ld_u32(blk + 12);
    uint32_t scw, mnw;   // 4 bytes: scales / mins of sub-blocks (c<2 ? 0..3 : 4..7)
    if (c < 2) {
        scw = Sw & 0x3f3f3f3fu;
        mnw = Mw & 0x3f3f3f3fu;
    } else {
        scw = (Xw & 0x0f0f0f0fu) | (((Sw >> 6) & 0x03030303u) << 4);
        mnw = ((Xw >> 4) & 0x0f0f0f0fu) | (((Mw >> 6) & 0x03030303u) << 4);
    }
    const int bsh = 16 * (c & 1);
    const int sc0 = (scw >> bsh) & 0xFF, sc1 = (scw >> (bsh + 8)) & 0xFF;
    const int mn0 = (mnw >> bsh) & 0xFF, mn1 = (mnw >> (bsh + 8)) & 0xFF;
    uint32_t lo[8], hi[8];
    if constexpr (TYPE == T_Q4_K) {
#pragma unroll
        for (int i = 0; i < 8; ++i) { lo[i] = qw[i] & 0x0F0F0F0Fu; hi[i] = (qw[i] >> 4) & 0x0F0F0F0Fu; }
    } else {
        uint32_t hw[8];
        ld_words_a4<8>(blk + 16, hw);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (qw[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c)) & 0x01010101u) << 4);
            hi[i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c + 1)) & 0x01010101u) << 4);
        }
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = reinterpret_cast<const int4 *>(A.q[m] + sb * 256 + 64 * c);
        const int4 a0 = aq[0], a1 = aq[1], a2 = aq[2], a3 = aq[3];
        int S0 = dp4a_us(lo[0], a0.x, 0);
        S0 = dp4a_us(lo[1], a0.y, S0);
        S0 = dp4a_us(lo[2], a0.z, S0);
        S0 = dp4a_us(lo[3], a0.w, S0);
        S0 = dp4a_us(lo[4], a1.x, S0);
        S0 = dp4a_us(lo[5], a1.y, S0);
        S0 = dp4a_us(lo[6], a1.z, S0);
        S0 = dp4a_us(lo[7], a1.w, S0);
        int S1 = dp4a_us(hi[0], a2.x, 0);
        S1 = dp4a_us(hi[1], a2.y, S1);
        S1 = dp4a_us(hi[2], a2.z, S1);
        S1 = dp4a_us(hi[3], a2.w, S1);
        S1 = dp4a_us(hi[4], a3.x, S1);
        S1 = dp4a_us(hi[5], a3.y, S1);
        S1 = dp4a_us(hi[6], a3.z, S1);
        S1 = dp4a_us(hi[7], a3.w, S1);
        const int2 bsv = *reinterpret_cast<const int2 *>(A.bs[m] + sb * 16 + 4 * c);
        const int A0 = bs_lo(bsv.x) + bs_hi(bsv.x), A1 = bs_lo(bsv.y) + bs_hi(bsv.y);
        if constexpr (ACT == ACT_CPU) {
            const int I = sc0 * S0 + sc1 * S1;
            const int Mi = mn0 * A0 + mn1 * A1;
            acc[m] += A.sc[m][sb] * (dm.x * static_cast<float>(I) - dm.y * static_cast<float>(Mi));
        } else {
            const float d80 = A.sc[m][sb * 8 + 2 * c], d81 = A.sc[m][sb * 8 + 2 * c + 1];
            const float fI = d80 * static_cast<float>(sc0 * S0) + d81 * static_cast<float>(sc1 * S1);
            const float fM = d80 * static_cast<float>(mn0 * A0) + d81 * static_cast<float>(mn1 * A1);
            acc[m] += dm.x * fI - dm.y * fM;
        }
    }
}

// Q6_K: task = (super-block, 128-element half n)
template <int ACT, int NMX>
__device__ __forceinline__ void task_q6_K(const uint8_t *row, int t, const Acts<NMX> &A, float (&acc)[NMX]) {
    const int sb = t >> 1, n = t & 1;
    const uint8_t *blk = row + sb * 210;
    uint32_t ql[16], qh[8], scw[2];
    ld_words_a2<16>(blk + 64 * n, ql);
    ld_words_a2<8>(blk + 128 + 32 * n, qh);
    ld_words_a2<2>(blk + 192 + 8 * n, scw);
    const float d = ld_half(blk + 208);
    uint32_t g[4][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        g[0][i] = (ql[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4);
        g[1][i] = (ql[8 + i] & 0x0F0F0F0Fu) | ((qh[i] << 2) & 0x30303030u);
        g[2][i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (qh[i] & 0x30303030u);
        g[3][i] = ((ql[8 + i] >> 4) & 0x0F0F0F0Fu) | ((qh[i] >> 2) & 0x30303030u);
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = reinterpret_cast<const int4 *>(A.q[m] + sb * 256 + 128 * n);
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + sb * 16 + 8 * n);
        const int bsw[4] = {bsv.x, bsv.y, bsv.z, bsv.w};
        int I = 0;
        float fI = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int4 a0 = aq[2 * k], a1 = aq[2 * k + 1];
            int S0 = dp4a_us(g[k][0], a0.x, 0);
            S0 = dp4a_us(g[k][1], a0.y, S0);
            S0 = dp4a_us(g[k][2], a0.z, S0);
            S0 = dp4a_us(g[k][3], a0.w, S0);
            int S1 = dp4a_us(g[k][4], a1.x, 0);
            S1 = dp4a_us(g[k][5], a1.y, S1);
            S1 = dp4a_us(g[k][6], a1.z, S1);
            S1 = dp4a_us(g[k][7], a1.w, S1);
            const uint32_t sw = scw[k >> 1];
            const int s0 = static_cast<int8_t>((sw >> (16 * (k & 1))) & 0xFF);
            const int s1 = static_cast<int8_t>((sw >> (16 * (k & 1) + 8)) & 0xFF);
            const int Ik = s0 * (S0 - 32 * bs_lo(bsw[k])) + s1 * (S1 - 32 * bs_hi(bsw[k]));
            if constexpr (ACT == ACT_CPU) I += Ik;
            else fI += A.sc[m][sb * 8 + 4 * n + k] * static_cast<float>(Ik);
        }
        if constexpr (ACT == ACT_CPU) acc[m] += A.sc[m][sb] * (d * static_cast<float>(I));
        else acc[m] += d * fI;
    }
}

template <int TYPE, int ACT, int NMX>
__device__ __forceinline__ void task_dot(const uint8_t *row, int t, const Acts<NMX> &A, float (&acc)[NMX]) {
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q5_0 || TYPE == T_Q8_0) task_legacy<TYPE, NMX>(row, t, A, acc);
    else if constexpr (TYPE == T_Q2_K) task_q2_K<ACT, NMX>(row, t, A, acc);
    else if constexpr (TYPE == T_Q3_K) task_q3_K<ACT, NMX>(row, t, A, acc);
    else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) task_q45_K<TYPE, ACT, NMX>(row, t, A, acc);
    else task_q6_K<ACT, NMX>(row, t, A, acc);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
struct GemvCtrl {
    int32_t x[GEMV_MAX_ENTRIES];          // expert of entry e = tok * nchannels_dst + pick
    int16_t first[GEMV_MAX_ENTRIES];
    int16_t uidx[GEMV_MAX_ENTRIES];
    int16_t eslot[GEMV_MAX_ENTRIES];      // activation slot of entry
    int16_t gmem[GEMV_MAX_ENTRIES];       // CSR members (entry ids)
    int32_t uexp[GEMV_MAX_ENTRIES];
    int16_t goff[GEMV_MAX_ENTRIES + 2];
    int16_t shslot[8];
    uint32_t keys[GEMV_MAX_KEYS];
    int32_t seg_g[GEMV_MAX_SEGMENTS], seg_r0[GEMV_MAX_SEGMENTS], seg_r1[GEMV_MAX_SEGMENTS];
    int32_t seg_t0[GEMV_MAX_SEGMENTS + 1];
    int32_t n_unique, n_seg, n_tiles, n_keys, fail;
};

template <int TYPE, int ACT, int NMX>
__global__ void __launch_bounds__(GEMV_THREADS, 1) moe_gemv_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    GemvCtrl &C = *reinterpret_cast<GemvCtrl *>(smem + 2 * GEMV_MAX_STAGES * 8);
    uint8_t *act_area = smem + a.ctrl_bytes;
    uint8_t *stage_area = act_area + static_cast<size_t>(a.act_slots) * a.slot_bytes;
    const uint32_t stage_bytes = a.part_bytes * static_cast<uint32_t>(a.n_parts);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nch = a.nchannels_dst;
    const int N = a.ncols_dst * nch;
    const bool has_shared = a.shared_up != nullptr;
    const int S = a.n_stages;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        fence_mbar_init();
        C.fail = 0;
    }
    __syncthreads();

    // ---- routed entries: validate and de-duplicate -------------------------
    for (int e = tid; e < N; e += blockDim.x) {
        const int t = e / nch, p = e % nch;
        const int x = a.ids[p + static_cast<int64_t>(t) * a.ids_stride];
        if (x < 0 || x >= a.n_experts) { C.fail = 1; set_error(a.err, DERR_BAD_ID); }
        C.x[e] = x;
    }
    __syncthreads();
    if (C.fail) return;
    for (int e = tid; e < N; e += blockDim.x) {
        int f = e;
        for (int j = 0; j < e; ++j) if (C.x[j] == C.x[e]) { f = j; break; }
        C.first[e] = static_cast<int16_t>(f);
    }
    __syncthreads();
    for (int e = tid; e < N; e += blockDim.x) {
        if (C.first[e] == e) {
            int u = 0;
            for (int j = 0; j < e; ++j) u += (C.first[j] == j);
            C.uidx[e] = static_cast<int16_t>(u);
            C.uexp[u] = C.x[e];
        }
    }
    __syncthreads();
    for (int e = tid; e < N; e += blockDim.x)
        if (C.first[e] != e) C.uidx[e] = C.uidx[C.first[e]];
    if (tid == 0) {
        int U = 0;
        for (int e = 0; e < N; ++e) U += (C.first[e] == e);
        C.n_unique = U;
    }
    __syncthreads();
    const int U = C.n_unique;
    for (int u = tid; u < U; u += blockDim.x) {
        int c = 0;
        for (int e = 0; e < N; ++e) c += (C.uidx[e] == u);
        C.goff[u + 1] = static_cast<int16_t>(c);
    }
    __syncthreads();
    if (tid == 0) {
        C.goff[0] = 0;
        for (int u = 0; u < U; ++u) C.goff[u + 1] = static_cast<int16_t>(C.goff[u] + C.goff[u + 1]);
    }
    __syncthreads();
    for (int u = tid; u < U; u += blockDim.x) {
        int k = C.goff[u];
        for (int e = 0; e < N; ++e) if (C.uidx[e] == u) C.gmem[k++] = static_cast<int16_t>(e);
    }

    // ---- bookkeeping of the reference kernel, first CTA only (:163-198) ---
    if (blockIdx.x == 0) {
        const uint32_t clk = a.clock ? *a.clock : 0u;
        for (int e = tid; e < N; e += blockDim.x) {
            const int x = C.x[e];
            if (a.tbl) {
                const bool host = (reinterpret_cast<uintptr_t>(a.tbl[x]) & 1u) != 0;
                if (a.stamps) a.stamps[x] = clk;
                if (a.stats) {
                    if (host) {
                        const uint32_t s = atomicAdd(a.stats, 1u);
                        if (s < a.log_cap) a.stats[GEMV_LOG_BASE + s] = (static_cast<uint32_t>(a.cache_id) << 12) | x;
                    } else {
                        atomicAdd(a.stats + 1, 1u);
                    }
                }
            }
            if (a.use_gate && a.tbl_gate) {
                const bool host = (reinterpret_cast<uintptr_t>(a.tbl_gate[x]) & 1u) != 0;
                if (a.stamps_gate) a.stamps_gate[x] = clk;
                if (a.stats) {
                    if (host) {
                        const uint32_t s = atomicAdd(a.stats, 1u);
                        if (s < a.log_cap)
                            a.stats[GEMV_LOG_BASE + s] = (static_cast<uint32_t>(a.cache_id_gate) << 12) | x;
                    } else {
                        atomicAdd(a.stats + 1, 1u);
                    }
                }
            }
        }
    }

    // ---- this CTA's slice of the row space: segments and tiles ------------
    const int groups = U + (has_shared ? 1 : 0);
    const int64_t Rt = static_cast<int64_t>(groups) * a.nrows;
    const int64_t r_begin = Rt * blockIdx.x / gridDim.x;
    const int64_t r_end = Rt * (blockIdx.x + 1) / gridDim.x;
    const int rpt = a.rows_per_tile;
    if (tid == 0) {
        int ns = 0, nt = 0;
        int64_t r = r_begin;
        while (r < r_end) {
            const int g = static_cast<int>(r / a.nrows);
            const int r0 = static_cast<int>(r - static_cast<int64_t>(g) * a.nrows);
            const int64_t g_end = static_cast<int64_t>(g + 1) * a.nrows;
            const int r1 = static_cast<int>((g_end < r_end ? g_end : r_end) - static_cast<int64_t>(g) * a.nrows);
            if (ns >= GEMV_MAX_SEGMENTS) { C.fail = 1; set_error(a.err, DERR_TOO_MANY_SEGMENTS); break; }
            C.seg_g[ns] = g; C.seg_r0[ns] = r0; C.seg_r1[ns] = r1; C.seg_t0[ns] = nt;
            nt += (r1 - r0 + rpt - 1) / rpt;
            ns++;
            r = static_cast<int64_t>(g) * a.nrows + r1;
        }
        C.seg_t0[ns] = nt;
        C.n_seg = ns;
        C.n_tiles = nt;
        // activation keys: (channel_y << 16 | token), KEY_SHARED for the shared block
        int nk = 0;
        for (int s = 0; s < ns && !C.fail; ++s) {
            const int g = C.seg_g[s];
            if (g < U) {
                for (int j = C.goff[g]; j < C.goff[g + 1]; ++j) {
                    const int e = C.gmem[j];
                    const int t = e / nch, p = e % nch;
                    const uint32_t key = (static_cast<uint32_t>(p % a.nchannels_y) << 16) | static_cast<uint32_t>(t);
                    int v = 0;
                    while (v < nk && C.keys[v] != key) ++v;
                    if (v == nk) {
                        if (nk >= a.act_slots || nk >= GEMV_MAX_KEYS) { C.fail = 1; set_error(a.err, DERR_TOO_MANY_KEYS); break; }
                        C.keys[nk++] = key;
                    }
                    C.eslot[e] = static_cast<int16_t>(v);
                }
            } else {
                for (int t = 0; t < a.ncols_dst; ++t) {
                    const uint32_t key = a.shared_y ? ((KEY_SHARED << 16) | static_cast<uint32_t>(t)) : static_cast<uint32_t>(t);
                    int v = 0;
                    while (v < nk && C.keys[v] != key) ++v;
                    if (v == nk) {
                        if (nk >= a.act_slots || nk >= GEMV_MAX_KEYS) { C.fail = 1; set_error(a.err, DERR_TOO_MANY_KEYS); break; }
                        C.keys[nk++] = key;
                    }
                    C.shslot[t] = static_cast<int16_t>(v);
                }
            }
        }
        C.n_keys = nk;
    }
    __syncthreads();
    if (C.fail) return;
    const int n_tiles = C.n_tiles, n_seg = C.n_seg;

    auto tile_coords = [&](int i, int &g, int &row0, int &nr) {
        int s = 0;
        while (s + 1 < n_seg && C.seg_t0[s + 1] <= i) ++s;
        g = C.seg_g[s];
        row0 = C.seg_r0[s] + (i - C.seg_t0[s]) * rpt;
        const int lim = C.seg_r1[s];
        nr = (lim - row0) < rpt ? (lim - row0) : rpt;
    };

    if (warp == GEMV_CONSUMER_WARPS) {
        // =========================== producer warp ===========================
        const uint64_t pol = l2_evict_first_policy();
        int issued = 0;
        for (int i = 0; i < n_tiles; ++i) {
            const int s = i % S;
            if (i >= S) {
                if (!mbar_wait_bounded(&empty[s], static_cast<uint32_t>((i / S - 1) & 1), a.timeout_ns)) {
                    if (lane == 0) set_error(a.err, DERR_TIMEOUT_EMPTY);
                    break;
                }
            }
            int g, row0, nr;
            tile_coords(i, g, row0, nr);
            const char *src[2] = {nullptr, nullptr};
            bool dev[2] = {true, true};
            bool host16[2] = {false, false};
            if (g < U) {
                const int x = C.uexp[g];
                const uintptr_t p = reinterpret_cast<uintptr_t>(a.tbl[x]);
                src[0] = reinterpret_cast<const char *>(p & ~static_cast<uintptr_t>(1));
                dev[0] = !(p & 1u) && a.tma_main;
                host16[0] = (p & 1u) && a.tma_main;
                if (a.use_gate) {
                    if (a.tbl_gate) {
                        const uintptr_t pg = reinterpret_cast<uintptr_t>(a.tbl_gate[x]);
                        src[1] = reinterpret_cast<const char *>(pg & ~static_cast<uintptr_t>(1));
                        dev[1] = !(pg & 1u) && a.tma_gate;
                        host16[1] = (pg & 1u) && a.tma_gate;
                    } else {
                        src[1] = a.gate_dense + static_cast<uint64_t>(x) * a.gate_expert_bytes;
                        dev[1] = a.tma_gate;
                    }
                }
            } else {
                src[0] = a.shared_up;
                src[1] = a.shared_gate;
                dev[0] = dev[1] = a.tma_shared;
            }
            uint8_t *stage = stage_area + static_cast<size_t>(s) * stage_bytes;
            uint32_t tx = 0;
            // plain-load copies first (host-tagged or unaligned sources)
            for (int pidx = 0; pidx < a.n_parts; ++pidx) {
                const char *sp = src[pidx] + static_cast<uint64_t>(row0) * a.row_bytes;
                const uint32_t bytes = static_cast<uint32_t>(nr) * a.row_bytes;
                uint8_t *dp = stage + pidx * a.part_bytes;
                const uintptr_t a0 = reinterpret_cast<uintptr_t>(sp) & ~static_cast<uintptr_t>(15);
                const uintptr_t a1 = (reinterpret_cast<uintptr_t>(sp) + bytes + 15u) & ~static_cast<uintptr_t>(15);
                if (dev[pidx]) {
                    tx += static_cast<uint32_t>(a1 - a0);
                } else if (host16[pidx]) {
                    // the same 16-byte aligned range a bulk copy would move (it
                    // stays inside the expert: 16-byte aligned base and size)
                    const uint4 *s4 = reinterpret_cast<const uint4 *>(a0);
                    uint4 *d4 = reinterpret_cast<uint4 *>(dp);
                    const uint32_t n4 = static_cast<uint32_t>(a1 - a0) / 16u;
                    for (uint32_t j = lane; j < n4; j += 32) d4[j] = s4[j];
                } else {
                    // 4-byte words when the source allows, else 2-byte units;
                    // both keep the copy inside [sp, sp + bytes)
                    const uintptr_t off = reinterpret_cast<uintptr_t>(sp) & 15u;
                    if (((reinterpret_cast<uintptr_t>(sp) | bytes) & 3u) == 0) {
                        const uint32_t *s32 = reinterpret_cast<const uint32_t *>(sp);
                        uint32_t *d32 = reinterpret_cast<uint32_t *>(dp + off);
                        for (uint32_t j = lane; j < bytes / 4; j += 32) d32[j] = s32[j];
                    } else {
                        const uint16_t *s16 = reinterpret_cast<const uint16_t *>(sp);
                        uint16_t *d16 = reinterpret_cast<uint16_t *>(dp + off);
                        for (uint32_t j = lane; j < bytes / 2; j += 32) d16[j] = s16[j];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&full[s], tx);
                for (int pidx = 0; pidx < a.n_parts; ++pidx) {
                    if (!dev[pidx]) continue;
                    const char *sp = src[pidx] + static_cast<uint64_t>(row0) * a.row_bytes;
                    const uint32_t bytes = static_cast<uint32_t>(nr) * a.row_bytes;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(sp) & ~static_cast<uintptr_t>(15);
                    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(sp) + bytes + 15u) & ~static_cast<uintptr_t>(15);
                    bulk_g2s(stage + pidx * a.part_bytes, reinterpret_cast<const void *>(a0), static_cast<uint32_t>(a1 - a0),
                             &full[s], pol);
                }
            }
            __syncwarp();
            issued = i + 1;
        }
        // drain: never leave a bulk copy in flight when the CTA exits
        const int first = issued > S ? issued - S : 0;
        for (int i = first; i < issued; ++i) {
            if (!mbar_wait_bounded(&full[i % S], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
                if (lane == 0) set_error(a.err, DERR_DRAIN);
                break;
            }
        }
        return;
    }

    // ============================ consumer warps =============================
    const int K = a.K;
    const uint32_t sb_bytes = a.slot_bytes;
    {
        // stage the activation vectors this CTA needs
        const int nk = C.n_keys;
        const bool q81 = (ACT == ACT_Q8_1);
        constexpr bool kq = is_kquant(TYPE);
        const int nb = q81 ? K / 32 : (kq ? K / 256 : K / 32);
        for (int job = warp; job < nk * nb; job += GEMV_CONSUMER_WARPS) {
            const int v = job / nb, b = job % nb;
            const uint32_t key = C.keys[v];
            const uint32_t kc = key >> 16;
            const int t = static_cast<int>(key & 0xFFFFu);
            uint8_t *slot = act_area + static_cast<size_t>(v) * sb_bytes;
            int8_t *q = reinterpret_cast<int8_t *>(slot);
            int16_t *bs = reinterpret_cast<int16_t *>(slot + K);
            float *sc = reinterpret_cast<float *>(slot + K + K / 8);
            int64_t off;
            const void *base;
            if (kc == KEY_SHARED) { base = a.shared_y; off = t * a.shared_y_stride_col; }
            else { base = a.y; off = static_cast<int64_t>(kc) * a.stride_channel_y + t * a.stride_col_y; }
            if (q81) {
                stage_q81_block(reinterpret_cast<const uint8_t *>(base) + off * 36, q, bs, sc, b, lane);
            } else if (kq) {
                stage_q8K_block(reinterpret_cast<const float *>(base) + off, q, bs, sc, b, lane);
            } else {
                stage_q80_block(reinterpret_cast<const float *>(base) + off, q, bs, sc, b, lane);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CONSUMER_WARPS * 32) : "memory");
    }

    const int L = a.lanes_per_row;
    const int RP = 32 / L;
    const int sub = lane % L, rr = lane / L;
    const int Tk = (K / fmt<TYPE>::qk) * fmt<TYPE>::tasks;
    const uint32_t rb = a.row_bytes;

    for (int i = warp; i < n_tiles; i += GEMV_CONSUMER_WARPS) {
        const int s = i % S;
        if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        int g, row0, nr;
        tile_coords(i, g, row0, nr);
        const uint8_t *stage = stage_area + static_cast<size_t>(s) * stage_bytes;
        // the tile's bytes start at (source address & 15) inside each part
        const char *srcs[2];
        if (g < U) {
            const int x = C.uexp[g];
            srcs[0] = reinterpret_cast<const char *>(reinterpret_cast<uintptr_t>(a.tbl[x]) & ~static_cast<uintptr_t>(1));
            if (a.use_gate)
                srcs[1] = a.tbl_gate ? reinterpret_cast<const char *>(reinterpret_cast<uintptr_t>(a.tbl_gate[x]) &
                                                                      ~static_cast<uintptr_t>(1))
                                     : a.gate_dense + static_cast<uint64_t>(x) * a.gate_expert_bytes;
            else
                srcs[1] = nullptr;
        } else {
            srcs[0] = a.shared_up;
            srcs[1] = a.shared_gate;
        }
        const uint8_t *up_rows =
            stage + ((reinterpret_cast<uintptr_t>(srcs[0]) + static_cast<uint64_t>(row0) * rb) & 15u);
        const uint8_t *gate_rows =
            a.use_gate ? stage + a.part_bytes + ((reinterpret_cast<uintptr_t>(srcs[1]) + static_cast<uint64_t>(row0) * rb) & 15u)
                       : nullptr;

        const int nmem = g < U ? (C.goff[g + 1] - C.goff[g]) : a.ncols_dst;
        for (int mc = 0; mc < nmem; mc += NMX) {
            Acts<NMX> A;
            A.nm = nmem - mc < NMX ? nmem - mc : NMX;
#pragma unroll
            for (int m = 0; m < NMX; ++m) {
                int v = 0;
                if (m < A.nm) v = g < U ? C.eslot[C.gmem[C.goff[g] + mc + m]] : C.shslot[mc + m];
                const uint8_t *slot = act_area + static_cast<size_t>(v) * sb_bytes;
                A.q[m] = reinterpret_cast<const int8_t *>(slot);
                A.bs[m] = reinterpret_cast<const int16_t *>(slot + K);
                A.sc[m] = reinterpret_cast<const float *>(slot + K + K / 8);
            }
            for (int rbase = 0; rbase < nr; rbase += RP) {
                const int r = rbase + rr;
                const bool valid = r < nr;
                float acc[NMX], accg[NMX];
#pragma unroll
                for (int m = 0; m < NMX; ++m) { acc[m] = 0.f; accg[m] = 0.f; }
                if (valid) {
                    const uint8_t *urow = up_rows + static_cast<size_t>(r) * rb;
                    for (int t = sub; t < Tk; t += L) task_dot<TYPE, ACT, NMX>(urow, t, A, acc);
                    if (a.use_gate) {
                        const uint8_t *grow = gate_rows + static_cast<size_t>(r) * rb;
                        for (int t = sub; t < Tk; t += L) task_dot<TYPE, ACT, NMX>(grow, t, A, accg);
                    }
                }
                for (int off = L >> 1; off >= 1; off >>= 1) {
#pragma unroll
                    for (int m = 0; m < NMX; ++m) {
                        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
                        if (a.use_gate) accg[m] += __shfl_xor_sync(0xffffffffu, accg[m], off);
                    }
                }
                if (valid && sub == 0) {
                    const int row = row0 + r;
#pragma unroll
                    for (int m = 0; m < NMX; ++m) {
                        if (m >= A.nm) break;
                        int x = 0, t, p = 0;
                        if (g < U) {
                            const int e = C.gmem[C.goff[g] + mc + m];
                            t = e / nch; p = e % nch; x = C.x[e];
                        } else {
                            t = mc + m;
                        }
                        float result = acc[m];
                        if (a.has_fusion) {
                            const int64_t bias_idx = static_cast<int64_t>(x) * a.stride_channel_dst + row;
                            if (a.x_bias) result += a.x_bias[bias_idx];
                            if (a.use_gate) {
                                float gv = accg[m];
                                if (a.gate_bias) gv += a.gate_bias[bias_idx];
                                result = glu_apply(a.glu_op, gv, result, a.glu_limit);
                            }
                        }
                        if (g < U) a.dst[p * a.stride_channel_dst + t * a.stride_col_dst + row] = result;
                        else a.shared_dst[t * a.shared_stride_col_dst + row] = result;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

}  // namespace moe
