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
//  * sixteen consumer warps dequantize in registers and run dp4a/dp2a integer
//    dots against activations staged once per CTA in shared memory, stored in
//    16-byte pieces interleaved across K-chunks so lanes working on different
//    chunks hit different banks; a fused gate/up pair shares its activation
//    loads; rows reduce with warp shuffles and the epilogue applies the
//    reference's bias / GLU / shared-expert fusion (:241-284);
//  * the first CTA does the reference's per-(pick, token) bookkeeping: stamps,
//    hit count and miss log (:163-198).
#pragma once
#include "moe_common.cuh"

namespace moe {

constexpr int GEMV_CONSUMER_WARPS = 16;
constexpr int GEMV_THREADS = 32 * (GEMV_CONSUMER_WARPS + 1);
constexpr int GEMV_MAX_ENTRIES = 256;    // ncols_dst * nchannels_dst
constexpr int GEMV_MAX_SEGMENTS = 32;
constexpr int GEMV_MAX_STAGES = 48;
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
    // routing; expert-parallel: ids are global, this tensor holds experts
    // [id_offset, id_offset + n_experts), and with skip_foreign the other ids
    // are left out (no output) instead of being errors
    const int32_t *ids;
    int64_t ids_stride;
    int32_t id_offset, skip_foreign;
    int32_t host_only;              // only picks whose table entry is host memory (others left out, no output)
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
    // n_tile_warps: consumer warps that take tiles (tile i -> warp i % n);
    // n_stages is a multiple of it, so every stage is always consumed by the
    // same warp and a warp never waits on a stage more than one phase ahead
    int32_t lanes_per_row, rows_per_tile, n_stages, n_parts, act_slots, n_tile_warps;
    uint32_t part_bytes, slot_bytes, ctrl_bytes;
    int32_t tma_main, tma_gate, tma_shared;
    int *err;
    uint64_t timeout_ns;
};

// ---------------------------------------------------------------------------
// Activations staged in shared memory, one slot per distinct input vector:
//   int8 q[K] in 16-byte pieces: piece p of K-chunk c at unit p * NC + c,
//        a chunk being the CE elements one task reads (NC = K / CE)
//   int16 bsum16[K/16] (natural order)
//   f32 scale[K/32]: per 32 (Q8_0 / Q8_1) or per 256 (Q8_K, first K/256)
// ---------------------------------------------------------------------------
template <int TYPE> struct chunk_of {
    static constexpr int CE = is_kquant(TYPE) ? ((TYPE == T_Q4_K || TYPE == T_Q5_K) ? 64 : 128) : 32;
};

template <int TYPE>
__device__ __forceinline__ uint32_t act_offset(int e, int NC) {
    constexpr int CE = chunk_of<TYPE>::CE;
    const int c = e / CE, o = e % CE;
    return static_cast<uint32_t>(((o >> 4) * NC + c) * 16 + (o & 15));
}

template <int NMX>
struct Acts {
    const int4 *q[NMX];       // piece units of the slot
    const int16_t *bs[NMX];
    const float *sc[NMX];
    int nm, NC;
};

__device__ __forceinline__ int bs_lo(int w) { return static_cast<int16_t>(w & 0xFFFF); }
__device__ __forceinline__ int bs_hi(int w) { return w >> 16; }

// f32 loads; CG: through L2 only (data another CTA of the same grid wrote)
template <bool CG> __device__ __forceinline__ float ld_f32(const float *p) { return CG ? __ldcg(p) : *p; }
template <bool CG> __device__ __forceinline__ float4 ld_f32x4(const float *p) {
    return CG ? __ldcg(reinterpret_cast<const float4 *>(p)) : *reinterpret_cast<const float4 *>(p);
}

// Lane l's values of a Q8_K block (256 f32 at xb): elements 4l..4l+3 and
// 128+4l..128+4l+3 (coalesced float4 loads when xb is 16-byte aligned).
template <bool CG>
__device__ __forceinline__ void load_q8K_vals(const float *xb, bool al16, int lane, float (&v)[8]) {
    if (al16) {
        const float4 u0 = ld_f32x4<CG>(xb + 4 * lane);
        const float4 u1 = ld_f32x4<CG>(xb + 128 + 4 * lane);
        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) { v[j] = ld_f32<CG>(xb + 4 * lane + j); v[4 + j] = ld_f32<CG>(xb + 128 + 4 * lane + j); }
    }
}

// Q8_K block b from the lane values of load_q8K_vals: llama.cpp
// quantize_row_q8_K_ref, bit-exact.
template <int TYPE>
__device__ __forceinline__ void quant_q8K_vals(const float (&v)[8], int8_t *q, int16_t *bs, float *sc, int b, int lane,
                                               int NC) {
    float amax = 0.f, mval = 0.f;
    int midx = 1 << 30;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int idx = j < 4 ? 4 * lane + j : 128 + 4 * lane + (j - 4);
        const float ax = fabsf(v[j]);
        if (ax > amax) { amax = ax; mval = v[j]; midx = idx; }   // ascending idx within the lane
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float ov = __shfl_xor_sync(0xffffffffu, mval, off);
        const int oi = __shfl_xor_sync(0xffffffffu, midx, off);
        if (oa > amax || (oa == amax && oi < midx)) { amax = oa; mval = ov; midx = oi; }
    }
    int qq[8];
    float d = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int j = 0; j < 8; ++j) qq[j] = 0;
    } else {
        const float iscale = -127.f / mval;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = nearest_int_dev(__fmul_rn(iscale, v[j]));
            qq[j] = r < 127 ? r : 127;
        }
        d = 1.f / iscale;
    }
    uint32_t w0 = 0, w1 = 0;
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        w0 |= (static_cast<uint32_t>(qq[j]) & 0xFFu) << (8 * j);
        w1 |= (static_cast<uint32_t>(qq[j + 4]) & 0xFFu) << (8 * j);
        s0 += qq[j];
        s1 += qq[j + 4];
    }
    const int e0 = b * 256 + 4 * lane, e1 = e0 + 128;
    *reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(q) + act_offset<TYPE>(e0, NC)) = w0;
    *reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(q) + act_offset<TYPE>(e1, NC)) = w1;
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    if ((lane & 3) == 0) {
        bs[b * 16 + (lane >> 2)] = static_cast<int16_t>(s0);
        bs[b * 16 + 8 + (lane >> 2)] = static_cast<int16_t>(s1);
    }
    if (lane == 0) sc[b] = d;
}

// Q8_K block (256 f32 at x + 256 b): llama.cpp quantize_row_q8_K_ref, bit-exact.
template <int TYPE, bool CG = false>
__device__ __forceinline__ void stage_q8K_block(const float *x, bool al16, int8_t *q, int16_t *bs, float *sc, int b,
                                                int lane, int NC) {
    float v[8];
    load_q8K_vals<CG>(x + b * 256, al16, lane, v);
    quant_q8K_vals<TYPE>(v, q, bs, sc, b, lane, NC);
}

// Q8_0 block b from lane l's value (element 32 b + l): llama.cpp
// quantize_row_q8_0_ref, bit-exact.
template <int TYPE>
__device__ __forceinline__ void quant_q80_val(float v, int8_t *q, int16_t *bs, float *sc, int b, int lane, int NC) {
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = amax / 127.f;
    const float id = d != 0.f ? 1.0f / d : 0.0f;
    const int qi = static_cast<int>(roundf(__fmul_rn(v, id)));
    q[act_offset<TYPE>(b * 32 + lane, NC)] = static_cast<int8_t>(qi);
    int s = qi;
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((lane & 15) == 0) bs[b * 2 + (lane >> 4)] = static_cast<int16_t>(s);
    if (lane == 0) sc[b] = __half2float(__float2half_rn(d));
}

template <int TYPE, bool CG = false>
__device__ __forceinline__ void stage_q80_block(const float *x, int8_t *q, int16_t *bs, float *sc, int b, int lane,
                                                int NC) {
    quant_q80_val<TYPE>(ld_f32<CG>(x + b * 32 + lane), q, bs, sc, b, lane, NC);
}

// Block b of an f32 activation vector into its slot with llama.cpp CPU
// semantics: Q8_K blocks for K-quant weights, Q8_0 blocks otherwise.
template <int TYPE, bool CG = false>
__device__ __forceinline__ void stage_f32_block(const float *xv, uint8_t *slot, int K, int b, int lane) {
    constexpr int CE = chunk_of<TYPE>::CE;
    int8_t *q = reinterpret_cast<int8_t *>(slot);
    int16_t *bs = reinterpret_cast<int16_t *>(slot + K);
    float *sc = reinterpret_cast<float *>(slot + K + K / 8);
    if constexpr (is_kquant(TYPE))
        stage_q8K_block<TYPE, CG>(xv, (reinterpret_cast<uintptr_t>(xv) & 15u) == 0, q, bs, sc, b, lane, K / CE);
    else
        stage_q80_block<TYPE, CG>(xv, q, bs, sc, b, lane, K / CE);
}

// Q8_1 block (36 bytes) as given: copy qs, scale = d, per-16 sums. For
// Q4_0 / Q5_0 weights the per-16 sums are not needed: the sum area holds the
// block's stored s instead (one f32 per block, the same K / 8 bytes), which
// llama.cpp's vec_dot_q4_0_q8_1 / vec_dot_q5_0_q8_1 use for the weights'
// offset.
template <int TYPE>
__device__ __forceinline__ void stage_q81_block(const uint8_t *yb, int8_t *q, int16_t *bs, float *sc, int b, int lane,
                                                int NC) {
    const uint8_t *blk = yb + static_cast<size_t>(b) * 36;
    int s = 0;
    if (lane < 8) {
        const uint32_t w = ld_u32(blk + 4 + 4 * lane);
        *reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(q) + act_offset<TYPE>(b * 32 + 4 * lane, NC)) = w;
        s = dp4a_ss(static_cast<int>(w), 0x01010101, 0);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q5_0) {
        if (lane == 0) reinterpret_cast<float *>(bs)[b] = ld_half(blk + 2);
    } else {
        if (lane == 0) bs[b * 2] = static_cast<int16_t>(s);
        if (lane == 4) bs[b * 2 + 1] = static_cast<int16_t>(s);
    }
    if (lane == 0) sc[b] = ld_half(blk);
}

// ---------------------------------------------------------------------------
// Per-type task dots. A task is a fixed K-slice of a weight row (one K-chunk).
// RL weight rows (the up and the gate row of one output row when fused) share
// the activation loads; the lane adds its contribution for every member
// vector m into acc[r][m].
// ---------------------------------------------------------------------------

// Q4_0 / Q5_0 / Q8_0: task = one 32-element block
template <int TYPE, int ACT, int NMX, int RL>
__device__ __forceinline__ void task_legacy(const uint8_t *const (&rows)[RL], int b, const Acts<NMX> &A,
                                            float (&acc)[RL][NMX]) {
    float dw[RL];
    uint32_t lo[RL][4], hi[RL][4], w8[RL][8];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const uint8_t *blk = rows[r] + b * fmt<TYPE>::bytes;
        dw[r] = ld_half(blk);
        if constexpr (TYPE == T_Q4_0) {
            uint32_t w[4];
            ld_words_a2<4>(blk + 2, w);
#pragma unroll
            for (int i = 0; i < 4; ++i) { lo[r][i] = w[i] & 0x0F0F0F0Fu; hi[r][i] = (w[i] >> 4) & 0x0F0F0F0Fu; }
        } else if constexpr (TYPE == T_Q5_0) {
            uint32_t w[5];
            ld_words_a2<5>(blk + 2, w);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo[r][i] = (w[1 + i] & 0x0F0F0F0Fu) | spread4_bit4(w[0] >> (4 * i));
                hi[r][i] = ((w[1 + i] >> 4) & 0x0F0F0F0Fu) | spread4_bit4(w[0] >> (16 + 4 * i));
            }
        } else {
            ld_words_a2<8>(blk + 2, w8[r]);
        }
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 a0 = A.q[m][b], a1 = A.q[m][A.NC + b];
        // Q8_1 with Q4_0 / Q5_0: the block's stored s (see stage_q81_block)
        constexpr bool S_OFF = ACT == ACT_Q8_1 && TYPE != T_Q8_0;
        const int bsw = *reinterpret_cast<const int *>(A.bs[m] + b * 2);
        const int asum = S_OFF ? 0 : bs_lo(bsw) + bs_hi(bsw);
        const float s8 = S_OFF ? reinterpret_cast<const float *>(A.bs[m])[b] : 0.f;
        const float d8 = A.sc[m][b];
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            int S;
            if constexpr (TYPE == T_Q8_0) {
                S = dp4a_ss(static_cast<int>(w8[r][0]), a0.x, 0);
                S = dp4a_ss(static_cast<int>(w8[r][1]), a0.y, S);
                S = dp4a_ss(static_cast<int>(w8[r][2]), a0.z, S);
                S = dp4a_ss(static_cast<int>(w8[r][3]), a0.w, S);
                S = dp4a_ss(static_cast<int>(w8[r][4]), a1.x, S);
                S = dp4a_ss(static_cast<int>(w8[r][5]), a1.y, S);
                S = dp4a_ss(static_cast<int>(w8[r][6]), a1.z, S);
                S = dp4a_ss(static_cast<int>(w8[r][7]), a1.w, S);
            } else {
                S = dp4a_us(lo[r][0], a0.x, 0);
                S = dp4a_us(lo[r][1], a0.y, S);
                S = dp4a_us(lo[r][2], a0.z, S);
                S = dp4a_us(lo[r][3], a0.w, S);
                S = dp4a_us(hi[r][0], a1.x, S);
                S = dp4a_us(hi[r][1], a1.y, S);
                S = dp4a_us(hi[r][2], a1.z, S);
                S = dp4a_us(hi[r][3], a1.w, S);
                if constexpr (!S_OFF) S -= (TYPE == T_Q4_0 ? 8 : 16) * asum;
            }
            // Q8_0 / Q8_K activations (CPU semantics): the exact integer sum,
            // offset taken off, times d_w d_a; Q8_1 activations with Q4_0 /
            // Q5_0 (llama.cpp's CUDA vec_dot_q{4,5}_0_q8_1):
            // d_w * (sumi * d_a - offset * s)
            if constexpr (S_OFF)
                acc[r][m] += dw[r] * (static_cast<float>(S) * d8 - (TYPE == T_Q4_0 ? 8.f : 16.f) * s8);
            else
                acc[r][m] += (dw[r] * d8) * static_cast<float>(S);
        }
    }
}

// Q2_K: task = (super-block, 128-element half n)
template <int ACT, int NMX, int RL>
__device__ __forceinline__ void task_q2_K(const uint8_t *const (&rows)[RL], int t, const Acts<NMX> &A,
                                          float (&acc)[RL][NMX]) {
    const int sb = t >> 1, n = t & 1;
    uint32_t q[RL][8], sw0[RL], sw1[RL], mw0[RL], mw1[RL];
    float2 dm[RL];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const uint8_t *blk = rows[r] + sb * 84;
        ld_words_a4<8>(blk + 16 + 32 * n, q[r]);
        sw0[r] = ld_u32(blk + 8 * n);
        sw1[r] = ld_u32(blk + 8 * n + 4);
        dm[r] = __half22float2(*reinterpret_cast<const __half2 *>(blk + 80));
        mw0[r] = (sw0[r] >> 4) & 0x0F0F0F0Fu;
        mw1[r] = (sw1[r] >> 4) & 0x0F0F0F0Fu;
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = A.q[m] + t;
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + t * 8);
        int Ih[RL];
        float fI[RL], fM[RL];
#pragma unroll
        for (int r = 0; r < RL; ++r) { Ih[r] = 0; fI[r] = 0.f; fM[r] = 0.f; }
#pragma unroll
        for (int k = 3; k >= 0; --k) {
            const uint32_t M = 0x03030303u << (2 * k);
            const int4 a0 = aq[(2 * k) * A.NC], a1 = aq[(2 * k + 1) * A.NC];
            const int bw = k == 0 ? bsv.x : k == 1 ? bsv.y : k == 2 ? bsv.z : bsv.w;
            float d8k = 0.f;
            if constexpr (ACT == ACT_Q8_1) d8k = A.sc[m][t * 4 + k];
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                int S0 = dp4a_us(q[r][0] & M, a0.x, 0);
                S0 = dp4a_us(q[r][1] & M, a0.y, S0);
                S0 = dp4a_us(q[r][2] & M, a0.z, S0);
                S0 = dp4a_us(q[r][3] & M, a0.w, S0);
                int S1 = dp4a_us(q[r][4] & M, a1.x, 0);
                S1 = dp4a_us(q[r][5] & M, a1.y, S1);
                S1 = dp4a_us(q[r][6] & M, a1.z, S1);
                S1 = dp4a_us(q[r][7] & M, a1.w, S1);
                const uint32_t sw = k < 2 ? sw0[r] : sw1[r];
                const int sc0 = (sw >> (16 * (k & 1))) & 0xF;
                const int sc1 = (sw >> (16 * (k & 1) + 8)) & 0xF;
                const int Ik = sc0 * S0 + sc1 * S1;   // 4^k times the true value (exact)
                if constexpr (ACT == ACT_CPU) {
                    Ih[r] = (k == 3) ? Ik : (Ih[r] >> 2) + Ik;
                } else {
                    const uint32_t mw = k < 2 ? mw0[r] : mw1[r];
                    const int Mk = (k & 1) ? dp2a_hi_su(bw, mw, 0) : dp2a_lo_su(bw, mw, 0);
                    fI[r] += d8k * static_cast<float>(Ik >> (2 * k));
                    fM[r] += d8k * static_cast<float>(Mk);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            if constexpr (ACT == ACT_CPU) {
                int Mi = dp2a_lo_su(bsv.x, mw0[r], 0);
                Mi = dp2a_hi_su(bsv.y, mw0[r], Mi);
                Mi = dp2a_lo_su(bsv.z, mw1[r], Mi);
                Mi = dp2a_hi_su(bsv.w, mw1[r], Mi);
                acc[r][m] += A.sc[m][sb] * (dm[r].x * static_cast<float>(Ih[r]) - dm[r].y * static_cast<float>(Mi));
            } else {
                acc[r][m] += dm[r].x * fI[r] - dm[r].y * fM[r];
            }
        }
    }
}

// Q3_K: task = (super-block, 128-element half n)
template <int ACT, int NMX, int RL>
__device__ __forceinline__ void task_q3_K(const uint8_t *const (&rows)[RL], int t, const Acts<NMX> &A,
                                          float (&acc)[RL][NMX]) {
    const int sb = t >> 1, n = t & 1;
    uint32_t qw[RL][8], hw[RL][8], SW0[RL], SW1[RL];
    float d[RL];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const uint8_t *blk = rows[r] + sb * 110;
        uint32_t sc3[3];
        ld_words_a2<8>(blk + 32 + 32 * n, qw[r]);
        ld_words_a2<8>(blk, hw[r]);
        ld_words_a2<3>(blk + 96, sc3);
        d[r] = ld_half(blk + 108);
        if (n == 0) {
            SW0[r] = (sc3[0] & 0x0F0F0F0Fu) | ((sc3[2] & 0x03030303u) << 4);
            SW1[r] = (sc3[1] & 0x0F0F0F0Fu) | (((sc3[2] >> 2) & 0x03030303u) << 4);
        } else {
            SW0[r] = ((sc3[0] >> 4) & 0x0F0F0F0Fu) | (((sc3[2] >> 4) & 0x03030303u) << 4);
            SW1[r] = ((sc3[1] >> 4) & 0x0F0F0F0Fu) | (((sc3[2] >> 6) & 0x03030303u) << 4);
        }
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = A.q[m] + t;
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + t * 8);
        int I[RL];
        float fI[RL];
#pragma unroll
        for (int r = 0; r < RL; ++r) { I[r] = 0; fI[r] = 0.f; }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int4 a0 = aq[(2 * k) * A.NC], a1 = aq[(2 * k + 1) * A.NC];
            const int bw = k == 0 ? bsv.x : k == 1 ? bsv.y : k == 2 ? bsv.z : bsv.w;
            const int hs = 4 * n + k;
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                uint32_t u[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    u[i] = ((qw[r][i] >> (2 * k)) & 0x03030303u) | (((hw[r][i] >> hs) & 0x01010101u) << 2);
                int S0 = dp4a_us(u[0], a0.x, 0);
                S0 = dp4a_us(u[1], a0.y, S0);
                S0 = dp4a_us(u[2], a0.z, S0);
                S0 = dp4a_us(u[3], a0.w, S0);
                int S1 = dp4a_us(u[4], a1.x, 0);
                S1 = dp4a_us(u[5], a1.y, S1);
                S1 = dp4a_us(u[6], a1.z, S1);
                S1 = dp4a_us(u[7], a1.w, S1);
                const uint32_t SW = k < 2 ? SW0[r] : SW1[r];
                const int s0 = static_cast<int>((SW >> (16 * (k & 1))) & 0xFF) - 32;
                const int s1 = static_cast<int>((SW >> (16 * (k & 1) + 8)) & 0xFF) - 32;
                const int Ik = s0 * (S0 - 4 * bs_lo(bw)) + s1 * (S1 - 4 * bs_hi(bw));
                if constexpr (ACT == ACT_CPU) I[r] += Ik;
                else fI[r] += A.sc[m][t * 4 + k] * static_cast<float>(Ik);
            }
        }
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            if constexpr (ACT == ACT_CPU) acc[r][m] += A.sc[m][sb] * (d[r] * static_cast<float>(I[r]));
            else acc[r][m] += d[r] * fI[r];
        }
    }
}

// Q4_K / Q5_K: task = (super-block, 64-element chunk c) = sub-blocks 2c, 2c+1
template <int TYPE, int ACT, int NMX, int RL>
__device__ __forceinline__ void task_q45_K(const uint8_t *const (&rows)[RL], int t, const Acts<NMX> &A,
                                           float (&acc)[RL][NMX]) {
    const int sb = t >> 2, c = t & 3;
    uint32_t lo[RL][8], hi[RL][8];
    int sc0[RL], sc1[RL], mn0[RL], mn1[RL];
    float2 dm[RL];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const uint8_t *blk = rows[r] + sb * fmt<TYPE>::bytes;
        uint32_t qw[8];
        ld_words_a4<8>(blk + (TYPE == T_Q4_K ? 16 : 48) + 32 * c, qw);
        dm[r] = __half22float2(*reinterpret_cast<const __half2 *>(blk));
        const uint32_t Sw = ld_u32(blk + 4), Mw = ld_u32(blk + 8), Xw = ld_u32(blk + 12);
        uint32_t scw, mnw;
        if (c < 2) {
            scw = Sw & 0x3f3f3f3fu;
            mnw = Mw & 0x3f3f3f3fu;
        } else {
            scw = (Xw & 0x0f0f0f0fu) | (((Sw >> 6) & 0x03030303u) << 4);
            mnw = ((Xw >> 4) & 0x0f0f0f0fu) | (((Mw >> 6) & 0x03030303u) << 4);
        }
        const int bsh = 16 * (c & 1);
        sc0[r] = (scw >> bsh) & 0xFF; sc1[r] = (scw >> (bsh + 8)) & 0xFF;
        mn0[r] = (mnw >> bsh) & 0xFF; mn1[r] = (mnw >> (bsh + 8)) & 0xFF;
        if constexpr (TYPE == T_Q4_K) {
#pragma unroll
            for (int i = 0; i < 8; ++i) { lo[r][i] = qw[i] & 0x0F0F0F0Fu; hi[r][i] = (qw[i] >> 4) & 0x0F0F0F0Fu; }
        } else {
            uint32_t hw[8];
            ld_words_a4<8>(blk + 16, hw);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                lo[r][i] = (qw[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c)) & 0x01010101u) << 4);
                hi[r][i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c + 1)) & 0x01010101u) << 4);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = A.q[m] + t;
        const int4 a0 = aq[0], a1 = aq[A.NC], a2 = aq[2 * A.NC], a3 = aq[3 * A.NC];
        const int2 bsv = *reinterpret_cast<const int2 *>(A.bs[m] + t * 4);
        const int A0 = bs_lo(bsv.x) + bs_hi(bsv.x), A1 = bs_lo(bsv.y) + bs_hi(bsv.y);
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            int S0 = dp4a_us(lo[r][0], a0.x, 0);
            S0 = dp4a_us(lo[r][1], a0.y, S0);
            S0 = dp4a_us(lo[r][2], a0.z, S0);
            S0 = dp4a_us(lo[r][3], a0.w, S0);
            S0 = dp4a_us(lo[r][4], a1.x, S0);
            S0 = dp4a_us(lo[r][5], a1.y, S0);
            S0 = dp4a_us(lo[r][6], a1.z, S0);
            S0 = dp4a_us(lo[r][7], a1.w, S0);
            int S1 = dp4a_us(hi[r][0], a2.x, 0);
            S1 = dp4a_us(hi[r][1], a2.y, S1);
            S1 = dp4a_us(hi[r][2], a2.z, S1);
            S1 = dp4a_us(hi[r][3], a2.w, S1);
            S1 = dp4a_us(hi[r][4], a3.x, S1);
            S1 = dp4a_us(hi[r][5], a3.y, S1);
            S1 = dp4a_us(hi[r][6], a3.z, S1);
            S1 = dp4a_us(hi[r][7], a3.w, S1);
            if constexpr (ACT == ACT_CPU) {
                const int I = sc0[r] * S0 + sc1[r] * S1;
                const int Mi = mn0[r] * A0 + mn1[r] * A1;
                acc[r][m] += A.sc[m][sb] * (dm[r].x * static_cast<float>(I) - dm[r].y * static_cast<float>(Mi));
            } else {
                const float d80 = A.sc[m][t * 2], d81 = A.sc[m][t * 2 + 1];
                const float fI = d80 * static_cast<float>(sc0[r] * S0) + d81 * static_cast<float>(sc1[r] * S1);
                const float fM = d80 * static_cast<float>(mn0[r] * A0) + d81 * static_cast<float>(mn1[r] * A1);
                acc[r][m] += dm[r].x * fI - dm[r].y * fM;
            }
        }
    }
}

// Q6_K: task = (super-block, 128-element half n)
template <int ACT, int NMX, int RL>
__device__ __forceinline__ void task_q6_K(const uint8_t *const (&rows)[RL], int t, const Acts<NMX> &A,
                                          float (&acc)[RL][NMX]) {
    const int sb = t >> 1, n = t & 1;
    uint32_t ql[RL][16], qh[RL][8], scw[RL][2];
    float d[RL];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const uint8_t *blk = rows[r] + sb * 210;
        ld_words_a2<16>(blk + 64 * n, ql[r]);
        ld_words_a2<8>(blk + 128 + 32 * n, qh[r]);
        ld_words_a2<2>(blk + 192 + 8 * n, scw[r]);
        d[r] = ld_half(blk + 208);
    }
#pragma unroll
    for (int m = 0; m < NMX; ++m) {
        if (m >= A.nm) break;
        const int4 *aq = A.q[m] + t;
        const int4 bsv = *reinterpret_cast<const int4 *>(A.bs[m] + t * 8);
        int I[RL];
        float fI[RL];
#pragma unroll
        for (int r = 0; r < RL; ++r) { I[r] = 0; fI[r] = 0.f; }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int4 a0 = aq[(2 * k) * A.NC], a1 = aq[(2 * k + 1) * A.NC];
            const int bw = k == 0 ? bsv.x : k == 1 ? bsv.y : k == 2 ? bsv.z : bsv.w;
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                uint32_t g[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (k == 0) g[i] = (ql[r][i] & 0x0F0F0F0Fu) | ((qh[r][i] & 0x03030303u) << 4);
                    else if (k == 1) g[i] = (ql[r][8 + i] & 0x0F0F0F0Fu) | ((qh[r][i] << 2) & 0x30303030u);
                    else if (k == 2) g[i] = ((ql[r][i] >> 4) & 0x0F0F0F0Fu) | (qh[r][i] & 0x30303030u);
                    else g[i] = ((ql[r][8 + i] >> 4) & 0x0F0F0F0Fu) | ((qh[r][i] >> 2) & 0x30303030u);
                }
                int S0 = dp4a_us(g[0], a0.x, 0);
                S0 = dp4a_us(g[1], a0.y, S0);
                S0 = dp4a_us(g[2], a0.z, S0);
                S0 = dp4a_us(g[3], a0.w, S0);
                int S1 = dp4a_us(g[4], a1.x, 0);
                S1 = dp4a_us(g[5], a1.y, S1);
                S1 = dp4a_us(g[6], a1.z, S1);
                S1 = dp4a_us(g[7], a1.w, S1);
                const uint32_t sw = scw[r][k >> 1];
                const int s0 = static_cast<int8_t>((sw >> (16 * (k & 1))) & 0xFF);
                const int s1 = static_cast<int8_t>((sw >> (16 * (k & 1) + 8)) & 0xFF);
                const int Ik = s0 * (S0 - 32 * bs_lo(bw)) + s1 * (S1 - 32 * bs_hi(bw));
                if constexpr (ACT == ACT_CPU) I[r] += Ik;
                else fI[r] += A.sc[m][t * 4 + k] * static_cast<float>(Ik);
            }
        }
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            if constexpr (ACT == ACT_CPU) acc[r][m] += A.sc[m][sb] * (d[r] * static_cast<float>(I[r]));
            else acc[r][m] += d[r] * fI[r];
        }
    }
}

template <int TYPE, int ACT, int NMX, int RL>
__device__ __forceinline__ void task_dot(const uint8_t *const (&rows)[RL], int t, const Acts<NMX> &A,
                                         float (&acc)[RL][NMX]) {
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q5_0 || TYPE == T_Q8_0) task_legacy<TYPE, ACT, NMX, RL>(rows, t, A, acc);
    else if constexpr (TYPE == T_Q2_K) task_q2_K<ACT, NMX, RL>(rows, t, A, acc);
    else if constexpr (TYPE == T_Q3_K) task_q3_K<ACT, NMX, RL>(rows, t, A, acc);
    else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) task_q45_K<TYPE, ACT, NMX, RL>(rows, t, A, acc);
    else task_q6_K<ACT, NMX, RL>(rows, t, A, acc);
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
    const char *usrc[GEMV_MAX_ENTRIES][2];   // weight source of each group (up/main, gate)
    uint8_t ukind[GEMV_MAX_ENTRIES][2];      // 0 bulk copy, 1 host 16-byte copy, 2 plain copy
    uint8_t uhost[GEMV_MAX_ENTRIES][2];      // host-tagged table entry
    int16_t goff[GEMV_MAX_ENTRIES + 2];
    int16_t shslot[8];
    uint32_t keys[GEMV_MAX_KEYS];
    int32_t seg_g[GEMV_MAX_SEGMENTS], seg_r0[GEMV_MAX_SEGMENTS], seg_r1[GEMV_MAX_SEGMENTS];
    int32_t seg_t0[GEMV_MAX_SEGMENTS + 1];
    uint32_t fmask[GEMV_MAX_ENTRIES / 32];    // first occurrences (block grouping)
    int16_t cnt[GEMV_MAX_ENTRIES];            // members per group / placement cursors
    uint32_t wpre[GEMV_MAX_ENTRIES + 2];      // prefix of rows x weight per group (weighted split)
    int32_t n_unique, n_seg, n_tiles, n_keys, fail;
};

// One consumer warp's pass over a tile (SW = 32), or one half-warp's
// (SW = 16: lanes 0-15 and 16-31 each run their own tile). Fused (use_gate):
// RL = 2 rows per lane are the up and the gate row of one output row;
// unfused: RL = 1.
template <int TYPE, int ACT, int NMX, int RL, int SW = 32>
__device__ __forceinline__ void consume_tile(const GemvArgs &a, const GemvCtrl &C, const uint8_t *up_rows,
                                             const uint8_t *gate_rows, int nr, int g, int U, int row0,
                                             const uint8_t *act_area, int lane, uint64_t *dst_tag = nullptr,
                                             uint64_t *shared_tag = nullptr, uint32_t tag = 0) {
    static_assert(SW == 32 || SW == 16, "whole or half warps");
    const unsigned mask = SW == 32 ? 0xffffffffu : (0xffffu << (lane & 16));
    const int sl = lane & (SW - 1);
    const int L = a.lanes_per_row;
    const int RP = SW / L;
    const int sub = sl % L, rr = sl / L;
    const int K = a.K;
    constexpr int CE = chunk_of<TYPE>::CE;
    const int Tk = (K / fmt<TYPE>::qk) * fmt<TYPE>::tasks;
    const uint32_t rb = a.row_bytes;
    const int nch = a.nchannels_dst;
    const int nmem = g < U ? (C.goff[g + 1] - C.goff[g]) : a.ncols_dst;
    for (int mc = 0; mc < nmem; mc += NMX) {
        Acts<NMX> A;
        A.nm = nmem - mc < NMX ? nmem - mc : NMX;
        A.NC = K / CE;
#pragma unroll
        for (int m = 0; m < NMX; ++m) {
            int v = 0;
            if (m < A.nm) v = g < U ? C.eslot[C.gmem[C.goff[g] + mc + m]] : C.shslot[mc + m];
            const uint8_t *slot = act_area + static_cast<size_t>(v) * a.slot_bytes;
            A.q[m] = reinterpret_cast<const int4 *>(slot);
            A.bs[m] = reinterpret_cast<const int16_t *>(slot + K);
            A.sc[m] = reinterpret_cast<const float *>(slot + K + K / 8);
        }
        for (int rbase = 0; rbase < nr; rbase += RP) {
            const int ri = rbase + rr;
            const bool ok = ri < nr;
            const uint8_t *wrows[RL];
            wrows[0] = up_rows + static_cast<size_t>(ok ? ri : 0) * rb;
            if constexpr (RL == 2) wrows[1] = gate_rows + static_cast<size_t>(ok ? ri : 0) * rb;
            float acc[RL][NMX];
#pragma unroll
            for (int r = 0; r < RL; ++r)
#pragma unroll
                for (int m = 0; m < NMX; ++m) acc[r][m] = 0.f;
            if (ok)
                for (int t = sub; t < Tk; t += L) task_dot<TYPE, ACT, NMX, RL>(wrows, t, A, acc);
            for (int off = L >> 1; off >= 1; off >>= 1) {
#pragma unroll
                for (int r = 0; r < RL; ++r)
#pragma unroll
                    for (int m = 0; m < NMX; ++m) acc[r][m] += __shfl_xor_sync(mask, acc[r][m], off);
            }
            if (!ok || sub != 0) continue;
            const int row = row0 + ri;
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
                float result = acc[0][m];
                if (a.has_fusion) {
                    const int64_t bias_idx = static_cast<int64_t>(x) * a.stride_channel_dst + row;
                    if (a.x_bias) result += a.x_bias[bias_idx];
                    if constexpr (RL == 2) {
                        float gv = acc[1][m];
                        if (a.gate_bias) gv += a.gate_bias[bias_idx];
                        result = glu_apply(a.glu_op, gv, result, a.glu_limit);
                    }
                }
                const int64_t o = g < U ? p * a.stride_channel_dst + t * a.stride_col_dst + row
                                        : t * a.shared_stride_col_dst + row;
                (g < U ? a.dst : a.shared_dst)[o] = result;
                // tagged copy (value, tag) in one 64-bit store: a reader that
                // sees the tag sees the value
                uint64_t *tp = g < U ? dst_tag : shared_tag;
                if (tp) st_relaxed_u64(tp + o, (static_cast<uint64_t>(tag) << 32) | __float_as_uint(result));
            }
        }
    }
}

// Weight sources of one tile: part p < n_parts holds rows
// [row0[p], row0[p] + nr[p]) of src[p], rb bytes each, and lands at
// stage + p * part_bytes + (its source address & 15). kind: 0 = bulk copy,
// 1 = host memory, copied with 16-byte loads, 2 = plain 4/2-byte copies
// (source not 16-byte aligned).
struct TileSrc {
    const char *src[2];
    int kind[2];
    int row0[2], nr[2];
    int n_parts;
    uint32_t rb, part_bytes;
};

// n4 16-byte units from host memory (read over the host link) into shared
// memory by one warp. A load from host memory takes microseconds, so each
// lane keeps HOST_COPY_DEPTH loads in flight (all of a batch's loads issue
// before its stores) instead of one load-store pair at a time.
#ifndef HOST_COPY_DEPTH
#define HOST_COPY_DEPTH 8
#endif
__device__ __forceinline__ void copy_host16(uint4 *d4, const uint4 *s4, uint32_t n4, int lane) {
    constexpr int U = HOST_COPY_DEPTH;
    for (uint32_t j0 = 0; j0 < n4; j0 += 32u * U) {
        uint4 v[U];
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const uint32_t j = j0 + static_cast<uint32_t>(lane) + 32u * q;
            if (j < n4) v[q] = s4[j];
        }
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const uint32_t j = j0 + static_cast<uint32_t>(lane) + 32u * q;
            if (j < n4) d4[j] = v[q];
        }
    }
}

// Waits until the copies of ring indexes [max(lo, end - S), end) have landed
// (the last S the producer issued): no bulk copy is then in flight.
__device__ __forceinline__ void drain_tiles(int end, int S, uint64_t *full, uint64_t timeout_ns, int *err, int lane,
                                            int lo = 0) {
    const int first = end - S > lo ? end - S : lo;
    for (int gi = first; gi < end; ++gi) {
        if (!mbar_wait_sleep(&full[gi % S], static_cast<uint32_t>((gi / S) & 1), drain_limit_ns(timeout_ns))) {
            if (lane == 0) set_error(err, DERR_DRAIN);
            break;
        }
    }
}

// The producer warp: streams tiles 0..n_tiles-1 through the S-stage ring
// (tile i -> ring index g = g0 + i -> stage g % S, phase g / S; g0 > 0 when
// the ring carries on from earlier tiles of a persistent kernel). Tiles are issued in rounds
// of up to min(32, S): within a round no tile reuses a stage of the same
// round, so every lane waits for its own stage and issues its own bulk copies.
// Tiles that need plain copies (host memory or unaligned sources) follow,
// one at a time, copied by the whole warp. With drain set, ends after every
// issued copy has landed, so no bulk copy is in flight when the CTA exits (a
// caller that streams on passes drain = false and calls drain_tiles once at
// the end). Returns the number of tiles issued (n_tiles unless a wait ran out).
template <class Describe>
__device__ __forceinline__ int produce_tiles(int n_tiles, int S, uint64_t *full, uint64_t *empty,
                                             uint8_t *stage_area, uint32_t stage_bytes, Describe describe,
                                             uint64_t timeout_ns, int *err, int lane, int g0 = 0,
                                             bool drain = true) {
    const uint64_t pol = l2_evict_first_policy();
    const int R = S < 32 ? S : 32;
    int issued = 0;
    bool ok = true;
    for (int base = 0; base < n_tiles && ok; base += R) {
        const int cnt = (n_tiles - base) < R ? (n_tiles - base) : R;
        bool plain_tile = false, lane_ok = true;
        TileSrc ts;
        const int gi = g0 + base + lane, s = gi % S;
        if (lane < cnt) {
            describe(base + lane, ts);
            plain_tile = ts.kind[0] != 0 || (ts.n_parts > 1 && ts.kind[1] != 0);
        }
        // each lane issues its bulk tile as soon as its stage is free (every
        // pending stage is probed per pass; between passes the warp sleeps on
        // the oldest), not when the whole round is free
        bool need = lane < cnt && !plain_tile;
        const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
        for (;;) {
            if (need && (gi < S || mbar_test_wait(&empty[s], static_cast<uint32_t>((gi / S - 1) & 1)))) {
                uint8_t *stage = stage_area + static_cast<size_t>(s) * stage_bytes;
                uintptr_t lo[2], hi[2];
                uint32_t tx = 0;
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    if (p >= ts.n_parts) break;
                    const uint32_t bytes = static_cast<uint32_t>(ts.nr[p]) * ts.rb;
                    const uintptr_t sp = reinterpret_cast<uintptr_t>(ts.src[p]) + static_cast<uint64_t>(ts.row0[p]) * ts.rb;
                    lo[p] = sp & ~static_cast<uintptr_t>(15);
                    hi[p] = (sp + bytes + 15u) & ~static_cast<uintptr_t>(15);
                    tx += static_cast<uint32_t>(hi[p] - lo[p]);
                }
                mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    if (p >= ts.n_parts) break;
                    bulk_g2s(stage + p * ts.part_bytes, reinterpret_cast<const void *>(lo[p]),
                             static_cast<uint32_t>(hi[p] - lo[p]), &full[s], pol);
                }
                need = false;
            }
            const unsigned pend = __ballot_sync(0xffffffffu, need);
            if (!pend) break;
            if (static_cast<uint64_t>(clock64()) - t0 > lim) {
                lane_ok = !need;
                break;
            }
            // sleep (in hardware) until the oldest pending stage is free
            if (lane == __ffs(pend) - 1) mbar_try_wait_hint(&empty[s], static_cast<uint32_t>((gi / S - 1) & 1), 20000u);
            __syncwarp();
        }
        if (__any_sync(0xffffffffu, !lane_ok)) {
            if (lane == 0) set_error(err, DERR_TIMEOUT_EMPTY);
            // this round's copies land before the producer gives up (the
            // caller's drain covers the rounds before it)
            if (lane < cnt && !plain_tile && lane_ok)
                mbar_wait_sleep(&full[s], static_cast<uint32_t>((gi / S) & 1), drain_limit_ns(timeout_ns));
            issued = base;
            ok = false;
            break;
        }
        unsigned pending = __ballot_sync(0xffffffffu, plain_tile);
        while (pending) {
            const int l = __ffs(pending) - 1;
            pending &= pending - 1u;
            const int i = base + l, gi = g0 + i, s = gi % S;
            if (gi >= S && !mbar_wait_sleep(&empty[s], static_cast<uint32_t>((gi / S - 1) & 1), timeout_ns)) {
                if (lane == 0) set_error(err, DERR_TIMEOUT_EMPTY);
                ok = false;
                break;
            }
            TileSrc ts;
            describe(i, ts);
            uint8_t *stage = stage_area + static_cast<size_t>(s) * stage_bytes;
            uint32_t tx = 0;
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                if (p >= ts.n_parts) break;
                const uint32_t bytes = static_cast<uint32_t>(ts.nr[p]) * ts.rb;
                const char *sp = ts.src[p] + static_cast<uint64_t>(ts.row0[p]) * ts.rb;
                uint8_t *dp = stage + p * ts.part_bytes;
                const uintptr_t a0 = reinterpret_cast<uintptr_t>(sp) & ~static_cast<uintptr_t>(15);
                const uintptr_t a1 = (reinterpret_cast<uintptr_t>(sp) + bytes + 15u) & ~static_cast<uintptr_t>(15);
                if (ts.kind[p] == 0) {
                    tx += static_cast<uint32_t>(a1 - a0);
                } else if (ts.kind[p] == 1) {
                    // the range a bulk copy would move (inside the expert:
                    // 16-byte aligned base and size), with 16-byte loads
                    copy_host16(reinterpret_cast<uint4 *>(dp), reinterpret_cast<const uint4 *>(a0),
                                static_cast<uint32_t>(a1 - a0) / 16u, lane);
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
            // generic-proxy writes to the stage are ordered before later
            // bulk-copy (async-proxy) writes to it
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    if (p >= ts.n_parts || ts.kind[p] != 0) continue;
                    const uint32_t bytes = static_cast<uint32_t>(ts.nr[p]) * ts.rb;
                    const char *sp = ts.src[p] + static_cast<uint64_t>(ts.row0[p]) * ts.rb;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(sp) & ~static_cast<uintptr_t>(15);
                    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(sp) + bytes + 15u) & ~static_cast<uintptr_t>(15);
                    bulk_g2s(stage + p * ts.part_bytes, reinterpret_cast<const void *>(a0), static_cast<uint32_t>(a1 - a0),
                             &full[s], pol);
                }
            }
            __syncwarp();
        }
        issued = base + cnt;
    }
    if (drain) drain_tiles(g0 + issued, S, full, timeout_ns, err, lane, g0);
    return issued;
}

// This CTA's contiguous share of the row space of n_groups groups of nrows
// rows (CTA b of G takes rows [b*q + min(b, rem), ...) with q, rem =
// divmod(rows, G)), cut at group boundaries into segments of rpt-row tiles.
// One thread; 32-bit arithmetic (launchers keep n_groups * nrows < 2^31).
__device__ __forceinline__ int build_segments(GemvCtrl &C, uint32_t n_groups, uint32_t nrows, int rpt, int *err) {
    const uint32_t Rt = n_groups * nrows;
    const uint32_t G = gridDim.x, bid = blockIdx.x;
    const uint32_t q = Rt / G, rem = Rt % G;
    const uint32_t r_begin = bid * q + (bid < rem ? bid : rem);
    const uint32_t r_end = r_begin + q + (bid < rem ? 1u : 0u);
    int ns = 0, nt = 0;
    uint32_t g = r_begin / nrows, r0 = r_begin - g * nrows;
    for (uint32_t left = r_end - r_begin; left > 0; ++g, r0 = 0) {
        const uint32_t r1 = (nrows - r0 < left) ? nrows : r0 + left;
        if (ns >= GEMV_MAX_SEGMENTS) { C.fail = 1; set_error(err, DERR_TOO_MANY_SEGMENTS); break; }
        C.seg_g[ns] = static_cast<int32_t>(g);
        C.seg_r0[ns] = static_cast<int32_t>(r0);
        C.seg_r1[ns] = static_cast<int32_t>(r1);
        C.seg_t0[ns] = nt;
        nt += (static_cast<int>(r1 - r0) + rpt - 1) / rpt;
        ns++;
        left -= r1 - r0;
    }
    C.seg_t0[ns] = nt;
    C.n_seg = ns;
    C.n_tiles = nt;
    return ns;
}

// Weighted variant: group g's rows cost w_g each (w_g = ceil(members / nmx),
// the shared group has `shared_members`), so a group many tokens picked is
// spread over more CTAs. Warp 0 writes the prefix C.wpre[g] = sum of
// nrows * w over groups before g (groups 0..U-1 routed, U the shared one).
__device__ __forceinline__ void group_weight_prefix(GemvCtrl &C, int U, bool has_shared, int shared_members,
                                                    uint32_t nrows, int nmx, int lane) {
    const int GA = U + (has_shared ? 1 : 0);
    constexpr int PER = (GEMV_MAX_ENTRIES + 2 + 31) / 32;
    uint32_t part[PER], sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int g = PER * lane + i;
        uint32_t w = 0;
        if (g < GA) {
            const int m = g < U ? C.goff[g + 1] - C.goff[g] : shared_members;
            w = static_cast<uint32_t>((m + nmx - 1) / nmx);
            if (w < 1) w = 1;
        }
        part[i] = w * nrows;
        sum += part[i];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
    }
    uint32_t run = incl - sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int g = PER * lane + i;
        if (g <= GA) C.wpre[g] = run;
        run += part[i];
    }
}

// This CTA's share of the weighted row space (one thread): row r of group g
// goes to CTA floor((wpre[g] + r w_g) G / W), so every CTA gets ~W/G of
// weight; cut into segments of rpt-row tiles. 64-bit products.
__device__ __forceinline__ int build_segments_weighted(GemvCtrl &C, int n_groups, uint32_t nrows, int rpt, int *err) {
    const uint64_t W = C.wpre[n_groups], G = gridDim.x, b = blockIdx.x;
    const uint64_t lo = b * W, hi = (b + 1) * W;
    // first group whose weight range reaches past lo
    int g0 = 0, g1 = n_groups;
    while (g0 < g1) {
        const int mid = (g0 + g1) >> 1;
        if (static_cast<uint64_t>(C.wpre[mid + 1]) * G <= lo) g0 = mid + 1;
        else g1 = mid;
    }
    int ns = 0, nt = 0;
    for (int g = g0; g < n_groups; ++g) {
        const uint64_t og = static_cast<uint64_t>(C.wpre[g]) * G;
        if (og >= hi) break;
        const uint64_t den = static_cast<uint64_t>((C.wpre[g + 1] - C.wpre[g]) / nrows) * G;
        uint64_t r0 = lo > og ? (lo - og + den - 1) / den : 0;
        uint64_t r1 = (hi - og + den - 1) / den;
        if (r0 > nrows) r0 = nrows;
        if (r1 > nrows) r1 = nrows;
        if (r1 <= r0) continue;
        if (ns >= GEMV_MAX_SEGMENTS) { C.fail = 1; set_error(err, DERR_TOO_MANY_SEGMENTS); break; }
        C.seg_g[ns] = g;
        C.seg_r0[ns] = static_cast<int32_t>(r0);
        C.seg_r1[ns] = static_cast<int32_t>(r1);
        C.seg_t0[ns] = nt;
        nt += (static_cast<int>(r1 - r0) + rpt - 1) / rpt;
        ns++;
    }
    C.seg_t0[ns] = nt;
    C.n_seg = ns;
    C.n_tiles = nt;
    return ns;
}

// Tile i of the segment list: group, first row, row count.
__device__ __forceinline__ void segment_tile(const GemvCtrl &C, int n_seg, int rpt, int i, int &g, int &row0, int &nr) {
    int s = 0;
    while (s + 1 < n_seg && C.seg_t0[s + 1] <= i) ++s;
    g = C.seg_g[s];
    row0 = C.seg_r0[s] + (i - C.seg_t0[s]) * rpt;
    const int lim = C.seg_r1[s];
    nr = (lim - row0) < rpt ? (lim - row0) : rpt;
}

// build_groups for N <= 32 entries by one warp (lane = its lane), without
// block barriers: __match_any_sync groups equal experts.
template <class XOf, class Resolve>
__device__ __forceinline__ void build_groups_warp(GemvCtrl &C, int N, int n_experts, XOf x_of, Resolve resolve,
                                                  int *err, int lane, bool skip_foreign = false) {
    int x = -1 - lane;
    bool bad = false, valid = false;
    if (lane < N) {
        const int xe = x_of(lane);
        const bool out = xe < 0 || xe >= n_experts;
        bad = out && !skip_foreign;
        valid = !out;
        C.x[lane] = out ? -1 : xe;      // -1: another GPU's expert
        if (!out) x = xe;
    }
    if (__ballot_sync(0xffffffffu, bad)) {
        if (lane == 0) { C.fail = 1; set_error(err, DERR_BAD_ID); }
    } else {
        const unsigned same = __match_any_sync(0xffffffffu, x);
        const int f = __ffs(same) - 1;
        const unsigned vmask = __ballot_sync(0xffffffffu, valid);
        const unsigned firsts = __ballot_sync(0xffffffffu, valid && f == lane);
        const int u = __popc(firsts & ((1u << f) - 1u));
        int pos = 0;
        for (int j = 0; j < N; ++j) {
            const int fj = __shfl_sync(0xffffffffu, f, j);
            pos += ((vmask >> j) & 1u) && ((fj < f) || (fj == f && j < lane));
        }
        if (valid) {
            C.first[lane] = static_cast<int16_t>(f);
            C.uidx[lane] = static_cast<int16_t>(u);
            C.gmem[pos] = static_cast<int16_t>(lane);
            if (f == lane) {
                C.uexp[u] = x;
                C.goff[u] = static_cast<int16_t>(pos);
                resolve(u, x);
            }
        }
        if (lane == 0) {
            C.n_unique = __popc(firsts);
            C.goff[__popc(firsts)] = static_cast<int16_t>(__popc(vmask));
        }
    }
}

// Groups the N routed entries by expert. x_of(e) gives entry e's expert;
// groups (distinct experts) are numbered in first-occurrence order, gmem lists
// each group's entries (CSR, offsets goff) and resolve(u, x) records group u's
// weight sources. Called by every thread of the block; ends with a block
// barrier. A bad expert id sets C.fail.
template <class XOf, class Resolve>
__device__ __forceinline__ void build_groups(GemvCtrl &C, int N, int n_experts, XOf x_of, Resolve resolve,
                                             int *err, bool skip_foreign = false) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (N <= 32) {
        if (warp == 0) build_groups_warp(C, N, n_experts, x_of, resolve, err, lane, skip_foreign);
    } else {
        // N <= GEMV_MAX_ENTRIES < blockDim.x: thread e holds entry e, so whole
        // warps hold consecutive entries. Five block barriers, no serial loops
        // over the entries.
        bool act = tid < N;     // a valid entry of this GPU's experts
        const bool wact = warp < (N + 31) / 32;
        int x = -1 - tid;
        if (act) {
            const int xe = x_of(tid);
            const bool out = xe < 0 || xe >= n_experts;
            if (out && !skip_foreign) { C.fail = 1; set_error(err, DERR_BAD_ID); }
            C.x[tid] = out ? -1 : xe;   // -1: another GPU's expert
            if (!out) x = xe;
            act = !out;
        }
        if (tid < GEMV_MAX_ENTRIES) C.cnt[tid] = 0;
        __syncthreads();
        const bool ok = !C.fail;
        int f = tid;
        if (ok && wact) {
            // first occurrence: inside the warp by match_any, else in earlier warps
            const unsigned same = __match_any_sync(0xffffffffu, x);
            f = 32 * warp + (__ffs(same) - 1);
            for (int j = 0; j < 32 * warp; ++j)
                if (C.x[j] == x) { f = j; break; }
            const unsigned fm = __ballot_sync(0xffffffffu, act && f == tid);
            if (lane == 0) C.fmask[warp] = fm;
            if (act) C.first[tid] = static_cast<int16_t>(f);
        }
        __syncthreads();
        if (ok && act) {
            // group = number of first occurrences before this entry's first
            const int wf = f >> 5;
            int u = __popc(C.fmask[wf] & ((1u << (f & 31)) - 1u));
            for (int w = 0; w < wf; ++w) u += __popc(C.fmask[w]);
            C.uidx[tid] = static_cast<int16_t>(u);
            if (f == tid) C.uexp[u] = x;
            atomicAdd(reinterpret_cast<int *>(&C.cnt[u & ~1]), (u & 1) ? 0x10000 : 1);
        }
        __syncthreads();
        if (ok && warp == 0) {
            // exclusive scan of the group sizes (8 groups per lane)
            int U = 0;
            for (int w = 0; w < (N + 31) / 32; ++w) U += __popc(C.fmask[w]);
            int part[8], sum = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int u = 8 * lane + i;
                part[i] = u < U ? C.cnt[u] : 0;
                sum += part[i];
            }
            int incl = sum;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += o;
            }
            const int total = __shfl_sync(0xffffffffu, incl, 31);   // valid entries
            int run = incl - sum;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int u = 8 * lane + i;
                if (u < U) {
                    C.goff[u] = static_cast<int16_t>(run);
                    C.cnt[u] = 0;
                }
                run += part[i];
            }
            if (lane == 0) {
                C.n_unique = U;
                C.goff[U] = static_cast<int16_t>(total);
            }
        }
        __syncthreads();
        if (ok) {
            if (tid < C.n_unique) resolve(tid, C.uexp[tid]);
            if (act) {
                // member slot inside the group; the order of a group's members
                // does not change any result
                const int u = C.uidx[tid];
                const int r = atomicAdd(reinterpret_cast<int *>(&C.cnt[u & ~1]), (u & 1) ? 0x10000 : 1);
                const int pos = (u & 1) ? (r >> 16) : (r & 0xFFFF);
                C.gmem[C.goff[u] + pos] = static_cast<int16_t>(tid);
            }
        }
    }
    __syncthreads();
}

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

    for (int s = tid; s < S; s += blockDim.x) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], 1);
    }
    if (tid < S) fence_mbar_init();
    if (tid == 0) C.fail = 0;
    __syncthreads();

    // ---- routed entries: validate, de-duplicate, resolve table entries ------
    // Entry e = tok * nchannels_dst + pick. Groups (distinct experts) are
    // numbered in first-occurrence order; gmem lists each group's entries
    // (CSR, offsets goff). usrc/ukind hold each group's weight sources.
    auto resolve = [&](int u, int x) {
        const uintptr_t p = reinterpret_cast<uintptr_t>(a.tbl[x]);
        C.usrc[u][0] = reinterpret_cast<const char *>(p & ~static_cast<uintptr_t>(1));
        C.ukind[u][0] = static_cast<uint8_t>((p & 1u) ? (a.tma_main ? 1 : 2) : (a.tma_main ? 0 : 2));
        C.uhost[u][0] = static_cast<uint8_t>(p & 1u);
        C.usrc[u][1] = nullptr;
        C.ukind[u][1] = 0;
        C.uhost[u][1] = 0;
        if (a.use_gate) {
            if (a.tbl_gate) {
                const uintptr_t pg = reinterpret_cast<uintptr_t>(a.tbl_gate[x]);
                C.usrc[u][1] = reinterpret_cast<const char *>(pg & ~static_cast<uintptr_t>(1));
                C.ukind[u][1] = static_cast<uint8_t>((pg & 1u) ? (a.tma_gate ? 1 : 2) : (a.tma_gate ? 0 : 2));
                C.uhost[u][1] = static_cast<uint8_t>(pg & 1u);
            } else {
                C.usrc[u][1] = a.gate_dense + static_cast<uint64_t>(x) * a.gate_expert_bytes;
                C.ukind[u][1] = static_cast<uint8_t>(a.tma_gate ? 0 : 2);
            }
        }
    };
    build_groups(
        C, N, a.n_experts,
        [&](int e) {
            const int x = a.ids[e % nch + static_cast<int64_t>(e / nch) * a.ids_stride] - a.id_offset;
            // host_only: a pick served from device memory (pool slot) is another path's
            return a.host_only && x >= 0 && x < a.n_experts && !(reinterpret_cast<uintptr_t>(a.tbl[x]) & 1u) ? -1 : x;
        },
        resolve, a.err, a.skip_foreign != 0 || a.host_only != 0);
    if (C.fail) return;
    const int U = C.n_unique;

    // ---- bookkeeping of the reference kernel, first CTA only (:163-198) ---
    if (blockIdx.x == 0) {
        const uint32_t clk = a.clock ? *a.clock : 0u;
        for (int e = tid; e < N; e += blockDim.x) {
            const int x = C.x[e];
            if (x < 0) continue;   // another GPU's expert
            const int u = C.uidx[e];
            if (a.tbl) {
                if (a.stamps) a.stamps[x] = clk;
                if (a.stats) {
                    if (C.uhost[u][0]) {
                        const uint32_t s = atomicAdd(a.stats, 1u);
                        if (s < a.log_cap) a.stats[GEMV_LOG_BASE + s] = (static_cast<uint32_t>(a.cache_id) << 12) | x;
                    } else {
                        atomicAdd(a.stats + 1, 1u);
                    }
                }
            }
            if (a.use_gate && a.tbl_gate) {
                if (a.stamps_gate) a.stamps_gate[x] = clk;
                if (a.stats) {
                    if (C.uhost[u][1]) {
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

    // ---- this CTA's slice of the row space (weighted by members per pass):
    //      segments and tiles --------------------------------------------------
    const int rpt = a.rows_per_tile;
    if (warp == 0) {
        group_weight_prefix(C, U, has_shared, a.ncols_dst, static_cast<uint32_t>(a.nrows), NMX, lane);
        __syncwarp();
    }
    if (tid == 0) {
        const int ns = build_segments_weighted(C, U + (has_shared ? 1 : 0), static_cast<uint32_t>(a.nrows), rpt, a.err);
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

    auto tile_coords = [&](int i, int &g, int &row0, int &nr) { segment_tile(C, n_seg, rpt, i, g, row0, nr); };
    // source of each part of group g's tiles; kind: 0 = bulk copy, 1 = host with
    // 16-byte plain copies, 2 = plain 4/2-byte copies (unaligned source)
    auto tile_sources = [&](int g, const char *&s0, const char *&s1, int &k0, int &k1) {
        if (g < U) {
            s0 = C.usrc[g][0];
            s1 = C.usrc[g][1];
            k0 = C.ukind[g][0];
            k1 = C.ukind[g][1];
        } else {
            s0 = a.shared_up;
            s1 = a.shared_gate;
            k0 = k1 = a.tma_shared ? 0 : 2;
        }
    };

    if (warp == GEMV_CONSUMER_WARPS) {
        // =========================== producer warp ===========================
        produce_tiles(
            n_tiles, S, full, empty, stage_area, stage_bytes,
            [&](int i, TileSrc &ts) {
                int g;
                tile_coords(i, g, ts.row0[0], ts.nr[0]);
                ts.row0[1] = ts.row0[0];
                ts.nr[1] = ts.nr[0];
                tile_sources(g, ts.src[0], ts.src[1], ts.kind[0], ts.kind[1]);
                ts.n_parts = a.n_parts;
                ts.rb = a.row_bytes;
                ts.part_bytes = a.part_bytes;
            },
            a.timeout_ns, a.err, lane);
        return;
    }

    // ============================ consumer warps =============================
    const int K = a.K;
    {
        // stage the activation vectors this CTA needs
        const int nk = C.n_keys;
        const bool q81 = (ACT == ACT_Q8_1);
        constexpr bool kq = is_kquant(TYPE);
        constexpr int CE = chunk_of<TYPE>::CE;
        const int NC = K / CE;
        const int nb = q81 ? K / 32 : (kq ? K / 256 : K / 32);
        for (int job = warp; job < nk * nb; job += GEMV_CONSUMER_WARPS) {
            const int v = job / nb, b = job % nb;
            const uint32_t key = C.keys[v];
            const uint32_t kc = key >> 16;
            const int t = static_cast<int>(key & 0xFFFFu);
            uint8_t *slot = act_area + static_cast<size_t>(v) * a.slot_bytes;
            int8_t *q = reinterpret_cast<int8_t *>(slot);
            int16_t *bs = reinterpret_cast<int16_t *>(slot + K);
            float *sc = reinterpret_cast<float *>(slot + K + K / 8);
            int64_t off;
            const void *base;
            if (kc == KEY_SHARED) { base = a.shared_y; off = t * a.shared_y_stride_col; }
            else { base = a.y; off = static_cast<int64_t>(kc) * a.stride_channel_y + t * a.stride_col_y; }
            if (q81) {
                stage_q81_block<TYPE>(reinterpret_cast<const uint8_t *>(base) + off * 36, q, bs, sc, b, lane, NC);
            } else if (kq) {
                const float *xv = reinterpret_cast<const float *>(base) + off;
                stage_q8K_block<TYPE>(xv, (reinterpret_cast<uintptr_t>(xv) & 15u) == 0, q, bs, sc, b, lane, NC);
            } else {
                stage_q80_block<TYPE>(reinterpret_cast<const float *>(base) + off, q, bs, sc, b, lane, NC);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CONSUMER_WARPS * 32) : "memory");
    }

    const int nw = a.n_tile_warps;
    for (int i = warp; i < n_tiles && warp < nw; i += nw) {
        const int s = i % S;
        if (!mbar_wait_sleep(&full[s], static_cast<uint32_t>((i / S) & 1), a.timeout_ns)) {
            if (lane == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            break;
        }
        int g, row0, nr;
        tile_coords(i, g, row0, nr);
        const uint8_t *stage = stage_area + static_cast<size_t>(s) * stage_bytes;
        const char *s0, *s1;
        int k0, k1;
        tile_sources(g, s0, s1, k0, k1);
        // each part's bytes start at (source address & 15) inside it
        const uint8_t *up_rows = stage + ((reinterpret_cast<uintptr_t>(s0) + static_cast<uint64_t>(row0) * a.row_bytes) & 15u);
        if (a.use_gate) {
            const uint8_t *gate_rows =
                stage + a.part_bytes + ((reinterpret_cast<uintptr_t>(s1) + static_cast<uint64_t>(row0) * a.row_bytes) & 15u);
            consume_tile<TYPE, ACT, NMX, 2>(a, C, up_rows, gate_rows, nr, g, U, row0, act_area, lane);
        } else {
            consume_tile<TYPE, ACT, NMX, 1>(a, C, up_rows, up_rows, nr, g, U, row0, act_area, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

}  // namespace moe
