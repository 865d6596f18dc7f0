// moe_aux.cu -- the small kernels around the MUL_MAT_ID GEMV:
//   * activation quantizers (Q8_0, Q8_1, Q8_K), bit-exact with llama.cpp
//     (CPU quantize_row_q8_0_ref / quantize_row_q8_K_ref, CUDA quantize_q8_1);
//   * routing: top-k over router logits plus softmax gating weights;
//   * the weighted combine of the per-pick down projections (+ shared expert);
//   * synthetic quantized weights for tests and benchmarks.
#include "moe_aux.h"
#include "moe_route.cuh"
#include "moe_common.cuh"

namespace moe {

// ---------------------------------------------------------------------------
// activation quantizers: one warp per block
// ---------------------------------------------------------------------------
__global__ void quantize_act_kernel(int act_type, const float *__restrict__ x, uint8_t *__restrict__ y,
                                    int64_t n_rows, int64_t n_cols) {
    const int lane = threadIdx.x & 31;
    const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int qk = act_type == T_Q8_K ? 256 : 32;
    const int64_t nb_row = n_cols / qk;
    if (warp_global >= n_rows * nb_row) return;
    const int64_t row = warp_global / nb_row, b = warp_global % nb_row;
    const float *xr = x + row * n_cols + b * qk;
    if (act_type == T_Q8_K) {
        uint8_t *blk = y + (row * nb_row + b) * 292;
        float v[8];
        float amax = 0.f, mval = 0.f;
        int midx = 1 << 30;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = xr[lane * 8 + j];
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
        int s = 0;
        float d = 0.f;
        if (amax != 0.f) {
            const float iscale = -127.f / mval;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int r = nearest_int_dev(__fmul_rn(iscale, v[j]));
                const int qv = r < 127 ? r : 127;
                blk[4 + lane * 8 + j] = static_cast<uint8_t>(static_cast<int8_t>(qv));
                s += qv;
            }
            d = 1.f / iscale;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) blk[4 + lane * 8 + j] = 0;
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if ((lane & 1) == 0) {
            const int16_t s16 = static_cast<int16_t>(s);
            memcpy(blk + 260 + 2 * (lane >> 1), &s16, 2);
        }
        if (lane == 0) memcpy(blk, &d, 4);
    } else if (act_type == T_Q8_0) {
        uint8_t *blk = y + (row * nb_row + b) * 34;
        const float v = xr[lane];
        float amax = fabsf(v);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        blk[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(v, id))));
        if (lane == 0) *reinterpret_cast<__half *>(blk) = __float2half_rn(d);   // 34-byte blocks: 2-aligned
    } else {   // Q8_1, llama.cpp CUDA quantize_q8_1 semantics
        uint8_t *blk = y + (row * nb_row + b) * 36;
        const float v = xr[lane];
        float amax = fabsf(v), sum = v;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
        }
        const float d = amax / 127.f;
        const int8_t q = amax == 0.0f ? 0 : static_cast<int8_t>(roundf(v / d));
        blk[4 + lane] = static_cast<uint8_t>(q);
        if (lane == 0)   // 36-byte blocks: 4-aligned
            *reinterpret_cast<__half2 *>(blk) = __halves2half2(__float2half_rn(d), __float2half_rn(sum));
    }
}

cudaError_t launch_quantize_act(int act_type, const float *x, void *y, int64_t n_rows, int64_t n_cols,
                                cudaStream_t st) {
    const int qk = act_type == T_Q8_K ? 256 : 32;
    const int64_t warps = n_rows * (n_cols / qk);
    if (warps == 0) return cudaSuccess;
    const int64_t blocks = (warps * 32 + 255) / 256;
    quantize_act_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(act_type, x, static_cast<uint8_t *>(y),
                                                                       n_rows, n_cols);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// routing: one warp per token. Selection on the logits (descending, ties to
// the lower expert id); weights = softmax over all experts at the picks.
// ---------------------------------------------------------------------------
__global__ void topk_softmax_kernel(const float *__restrict__ logits, int n_experts, int k, int norm_w,
                                    int32_t *__restrict__ ids, float *__restrict__ weights) {
    const int t = blockIdx.x;
    route_token_warp(logits + static_cast<int64_t>(t) * n_experts, n_experts, k, norm_w, threadIdx.x,
                     ids + static_cast<int64_t>(t) * k, weights + static_cast<int64_t>(t) * k);
}

cudaError_t launch_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts, int64_t k, int norm_w,
                                int32_t *ids, float *weights, cudaStream_t st) {
    if (n_tok == 0) return cudaSuccess;
    topk_softmax_kernel<<<static_cast<unsigned>(n_tok), 32, 0, st>>>(logits, static_cast<int>(n_experts),
                                                                      static_cast<int>(k), norm_w, ids, weights);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// GLU pass for gate/up computed by separate GEMVs: the same glu_apply as the
// fused epilogue (reference kernels/moe-cache.cu:264-280)
// ---------------------------------------------------------------------------
__global__ void glu_kernel(const float *__restrict__ g, float *__restrict__ u, int64_t n, int op, float limit) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) u[i] = glu_apply(op, g[i], u[i], limit);
}

cudaError_t launch_glu(const float *g, float *u, int64_t n, int op, float limit, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    glu_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(g, u, n, op, limit);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// combine: out[t][r] = sum_p w[t][p] * y[t][p][r] (pick order) + ys[t][r]
// ---------------------------------------------------------------------------
__global__ void combine_kernel(const float *__restrict__ y, const float *__restrict__ w, const float *__restrict__ ys,
                               float *__restrict__ out, int H, int k) {
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= H) return;
    const float *yt = y + static_cast<int64_t>(t) * k * H;
    float acc = 0.f;
    for (int p = 0; p < k; ++p) {
        const float v = __fmul_rn(yt[static_cast<int64_t>(p) * H + r], w[t * k + p]);
        acc = p == 0 ? v : __fadd_rn(acc, v);
    }
    if (ys) acc = __fadd_rn(acc, ys[static_cast<int64_t>(t) * H + r]);
    out[static_cast<int64_t>(t) * H + r] = acc;
}

__global__ void combine_local_kernel(const float *__restrict__ y, const float *__restrict__ w,
                                     const float *__restrict__ ys, const int32_t *__restrict__ ids, int id_lo,
                                     int n_local, float *__restrict__ out, int H, int k) {
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= H) return;
    const float *yt = y + static_cast<int64_t>(t) * k * H;
    float acc = 0.f;
    bool any = false;
    for (int p = 0; p < k; ++p) {
        const int x = ids[t * k + p] - id_lo;
        if (x < 0 || x >= n_local) continue;
        const float v = __fmul_rn(yt[static_cast<int64_t>(p) * H + r], w[t * k + p]);
        acc = any ? __fadd_rn(acc, v) : v;
        any = true;
    }
    if (ys) acc = __fadd_rn(acc, ys[static_cast<int64_t>(t) * H + r]);
    out[static_cast<int64_t>(t) * H + r] = acc;
}

cudaError_t launch_combine_local(const float *y, const float *w, const float *ys, const int32_t *ids, int id_lo,
                                 int n_local, float *out, int64_t n_tok, int64_t H, int64_t k, cudaStream_t st) {
    if (n_tok == 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((H + 255) / 256), static_cast<unsigned>(n_tok));
    combine_local_kernel<<<grid, 256, 0, st>>>(y, w, ys, ids, id_lo, n_local, out, static_cast<int>(H),
                                                static_cast<int>(k));
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *y, const float *w, const float *ys, float *out, int64_t n_tok, int64_t H,
                           int64_t k, cudaStream_t st) {
    if (n_tok == 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((H + 255) / 256), static_cast<unsigned>(n_tok));
    combine_kernel<<<grid, 256, 0, st>>>(y, w, ys, out, static_cast<int>(H), static_cast<int>(k));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// synthetic quantized weights: N(0, sigma) from a counter hash, quantized with
// the same min/max algorithm as the CPU oracle's weight quantizer.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t h = mix64(seed ^ mix64(i));
    const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ float half_round(float f) { return __half2float(__float2half_rn(f)); }
__device__ __forceinline__ void put_half(uint8_t *p, float f) {
    const __half h = __float2half_rn(f);
    memcpy(p, &h, 2);
}

__device__ float signed_absmax_dev(const float *x, int n) {
    float amax = 0.f, mx = 0.f;
    for (int j = 0; j < n; ++j)
        if (amax < fabsf(x[j])) { amax = fabsf(x[j]); mx = x[j]; }
    return mx;
}

__device__ void fit_asym_dev(const float *x, int nsub, int sl, int qmax, int smax, float *d_out, float *dmin_out,
                             int *sc, int *mn, uint8_t *q) {
    float scale[16], off[16], maxs = 0, maxm = 0;
    for (int s = 0; s < nsub; ++s) {
        float lo = 0.f, hi = 0.f;
        for (int l = 0; l < sl; ++l) {
            const float v = x[s * sl + l];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        scale[s] = (hi - lo) / qmax;
        off[s] = -lo;
        maxs = fmaxf(maxs, scale[s]);
        maxm = fmaxf(maxm, off[s]);
    }
    const float d = half_round(maxs / smax), dmin = half_round(maxm / smax);
    for (int s = 0; s < nsub; ++s) {
        sc[s] = d > 0 ? clampi(__float2int_rn(scale[s] / d), 0, smax) : 0;
        mn[s] = dmin > 0 ? clampi(__float2int_rn(off[s] / dmin), 0, smax) : 0;
        const float dl = d * sc[s], ml = dmin * mn[s];
        for (int l = 0; l < sl; ++l)
            q[s * sl + l] = static_cast<uint8_t>(dl > 0 ? clampi(__float2int_rn((x[s * sl + l] + ml) / dl), 0, qmax) : 0);
    }
    *d_out = d;
    *dmin_out = dmin;
}

__device__ void fit_sym_dev(const float *x, int nsub, int sl, int qneg, int smax, float *d_out, int *sc, int8_t *q) {
    float scale[16], maxs = 0;
    for (int s = 0; s < nsub; ++s) {
        scale[s] = signed_absmax_dev(x + s * sl, sl) / -qneg;
        maxs = fmaxf(maxs, fabsf(scale[s]));
    }
    const float d = half_round(maxs / smax);
    for (int s = 0; s < nsub; ++s) {
        sc[s] = d > 0 ? clampi(__float2int_rn(scale[s] / d), -smax - 1, smax) : 0;
        const float dl = d * sc[s];
        for (int l = 0; l < sl; ++l)
            q[s * sl + l] = static_cast<int8_t>(dl != 0 ? clampi(__float2int_rn(x[s * sl + l] / dl), -qneg, qneg - 1) : 0);
    }
    *d_out = d;
}

__global__ void fill_quantized_kernel(int type, uint8_t *__restrict__ dst, int64_t n_blocks, int qk, int tsize,
                                      uint64_t seed, float sigma) {
    const int64_t ib = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (ib >= n_blocks) return;
    float x[256];
    for (int j = 0; j < qk; ++j) x[j] = sigma * normal_at(seed, static_cast<uint64_t>(ib) * qk + j);
    uint8_t y[210];
    for (int j = 0; j < tsize; ++j) y[j] = 0;
    switch (type) {
        case T_Q4_0: case T_Q5_0: {
            const int q5 = type == T_Q5_0;
            const float mx = signed_absmax_dev(x, 32);
            const float d = mx / (q5 ? -16.f : -8.f);
            const float id = d != 0.f ? 1.0f / d : 0.0f;
            put_half(y, d);
            uint32_t qh = 0;
            for (int j = 0; j < 16; ++j) {
                const float x0 = x[j] * id, x1 = x[16 + j] * id;
                const int xi0 = clampi(static_cast<int8_t>(x0 + (q5 ? 16.5f : 8.5f)), -128, q5 ? 31 : 15);
                const int xi1 = clampi(static_cast<int8_t>(x1 + (q5 ? 16.5f : 8.5f)), -128, q5 ? 31 : 15);
                y[(q5 ? 6 : 2) + j] = static_cast<uint8_t>((xi0 & 0xF) | ((xi1 & 0xF) << 4));
                qh |= ((static_cast<uint32_t>(xi0) & 0x10u) >> 4) << j;
                qh |= ((static_cast<uint32_t>(xi1) & 0x10u) >> 4) << (j + 16);
            }
            if (q5) memcpy(y + 2, &qh, 4);
        } break;
        case T_Q8_0: {
            float amax = 0.f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
            const float d = amax / 127.f, id = d != 0.f ? 1.0f / d : 0.0f;
            put_half(y, d);
            for (int j = 0; j < 32; ++j) y[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(roundf(x[j] * id)));
        } break;
        case T_Q2_K: {
            float d, dmin; int sc[16], mn[16]; uint8_t q[256];
            fit_asym_dev(x, 16, 16, 3, 15, &d, &dmin, sc, mn, q);
            for (int s = 0; s < 16; ++s) y[s] = static_cast<uint8_t>(sc[s] | (mn[s] << 4));
            for (int i = 0; i < 256; ++i) y[16 + (i / 128) * 32 + i % 32] |= static_cast<uint8_t>(q[i] << (2 * ((i % 128) / 32)));
            put_half(y + 80, d);
            put_half(y + 82, dmin);
        } break;
        case T_Q3_K: {
            float d; int sc[16]; int8_t q[256];
            fit_sym_dev(x, 16, 16, 4, 31, &d, sc, q);
            for (int i = 0; i < 256; ++i) {
                const int n = i / 128, s = (i % 128) / 32, l = i % 32, u = q[i] + 4;
                y[32 + n * 32 + l] |= static_cast<uint8_t>((u & 3) << (2 * s));
                if (u & 4) y[l] |= static_cast<uint8_t>(1u << (n * 4 + s));
            }
            for (int k = 0; k < 16; ++k) {
                const int v = sc[k] + 32;
                if (k < 8) y[96 + k] |= static_cast<uint8_t>(v & 0xF);
                else y[96 + k - 8] |= static_cast<uint8_t>((v & 0xF) << 4);
                y[104 + (k % 4)] |= static_cast<uint8_t>((v >> 4) << (2 * (k / 4)));
            }
            put_half(y + 108, d);
        } break;
        case T_Q4_K: case T_Q5_K: {
            const int five = type == T_Q5_K;
            float d, dmin; int sc[8], mn[8]; uint8_t q[256];
            fit_asym_dev(x, 8, 32, five ? 31 : 15, 63, &d, &dmin, sc, mn, q);
            put_half(y, d);
            put_half(y + 2, dmin);
            for (int j = 0; j < 4; ++j) {
                y[4 + j] = static_cast<uint8_t>(sc[j] | ((sc[j + 4] >> 4) << 6));
                y[8 + j] = static_cast<uint8_t>(mn[j] | ((mn[j + 4] >> 4) << 6));
                y[12 + j] = static_cast<uint8_t>((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
            }
            uint8_t *qs = y + (five ? 48 : 16);
            for (int c = 0; c < 4; ++c)
                for (int l = 0; l < 32; ++l) {
                    const int lo = q[64 * c + l], hi = q[64 * c + 32 + l];
                    qs[32 * c + l] = static_cast<uint8_t>((lo & 0xF) | ((hi & 0xF) << 4));
                    if (five) {
                        y[16 + l] |= static_cast<uint8_t>(((lo >> 4) & 1) << (2 * c));
                        y[16 + l] |= static_cast<uint8_t>(((hi >> 4) & 1) << (2 * c + 1));
                    }
                }
        } break;
        case T_Q6_K: {
            float d; int sc[16]; int8_t q[256];
            fit_sym_dev(x, 16, 16, 32, 127, &d, sc, q);
            for (int n = 0; n < 2; ++n)
                for (int l = 0; l < 32; ++l) {
                    const int b = 128 * n;
                    const int q1 = q[b + l] + 32, q2 = q[b + 32 + l] + 32, q3 = q[b + 64 + l] + 32, q4 = q[b + 96 + l] + 32;
                    y[64 * n + l] = static_cast<uint8_t>((q1 & 0xF) | ((q3 & 0xF) << 4));
                    y[64 * n + 32 + l] = static_cast<uint8_t>((q2 & 0xF) | ((q4 & 0xF) << 4));
                    y[128 + 32 * n + l] =
                        static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
                }
            for (int s = 0; s < 16; ++s) y[192 + s] = static_cast<uint8_t>(static_cast<int8_t>(sc[s]));
            put_half(y + 208, d);
        } break;
        default: break;
    }
    uint8_t *out = dst + ib * tsize;
    for (int j = 0; j < tsize; ++j) out[j] = y[j];
}

cudaError_t launch_fill_quantized(int type, void *dst, int64_t n_rows, int64_t n_cols, uint64_t seed, float sigma,
                                  cudaStream_t st) {
    int qk, ts;
    switch (type) {
        case T_Q4_0: qk = 32; ts = 18; break;
        case T_Q5_0: qk = 32; ts = 22; break;
        case T_Q8_0: qk = 32; ts = 34; break;
        case T_Q2_K: qk = 256; ts = 84; break;
        case T_Q3_K: qk = 256; ts = 110; break;
        case T_Q4_K: qk = 256; ts = 144; break;
        case T_Q5_K: qk = 256; ts = 176; break;
        case T_Q6_K: qk = 256; ts = 210; break;
        default: return cudaErrorInvalidValue;
    }
    const int64_t nb = n_rows * (n_cols / qk);
    if (nb == 0) return cudaSuccess;
    fill_quantized_kernel<<<static_cast<unsigned>((nb + 127) / 128), 128, 0, st>>>(
        type, static_cast<uint8_t *>(dst), nb, qk, ts, seed, sigma);
    return cudaGetLastError();
}

}  // namespace moe
