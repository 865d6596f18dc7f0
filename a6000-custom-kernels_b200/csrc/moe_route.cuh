// moe_route.cuh -- top-k routing of one token by one warp, shared by the
// stand-alone routing kernel and the fused layer kernel so both give the same
// bits. It restates llama.cpp's MoE gating (build_moe_ffn: softmax over the
// router logits, argsort top-k, optional renormalisation over the k picks).
#pragma once
#include <cmath>
#include <cstdint>

namespace moe {

// Running best of a scan: the first candidate is always taken (even -inf or
// NaN), later ones when larger, ties to the lower expert id.
__device__ __forceinline__ bool route_better(float v, int e, float bv, int bi) {
    return bi == 0x7fffffff || v > bv || (v == bv && e < bi);
}

// Top-k of one token's logits l[0..n_experts) (descending, ties to the lower
// expert id) and gating weights expf(l - max) / sum_e expf(l_e - max), where
// the sum runs lane-strided (lane j adds experts j, j + 32, ...) and then over
// the lanes by xor butterfly; with norm_w the k weights are divided by their
// sum in pick order. Lane 0 writes ids[0..k) and w[0..k). All 32 lanes call.
__device__ __forceinline__ void route_token_warp(const float *__restrict__ l, int n_experts, int k, int norm_w,
                                                 int lane, int32_t *ids, float *w) {
    constexpr int REG = 32;   // logits per lane held in registers (n_experts <= 1024)
    if (n_experts <= 32 * REG) {
        float v[REG];
#pragma unroll
        for (int j = 0; j < REG; ++j) {
            const int e = lane + 32 * j;
            v[j] = e < n_experts ? l[e] : 0.f;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < REG; ++j)
            if (lane + 32 * j < n_experts) mx = fmaxf(mx, v[j]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < REG; ++j)
            if (lane + 32 * j < n_experts) sum += expf(v[j] - mx);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        uint32_t taken = 0;
        float ws = 0.f;
        for (int q = 0; q < k; ++q) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < REG; ++j) {
                const int e = lane + 32 * j;
                if (e < n_experts && !((taken >> j) & 1u) && route_better(v[j], e, bv, bi)) { bv = v[j]; bi = e; }
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (oi != 0x7fffffff && route_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (bi != 0x7fffffff && (bi & 31) == lane) taken |= 1u << (bi >> 5);
            if (lane == 0) {
                const float wq = expf(bv - mx) / sum;
                ids[q] = bi;
                w[q] = wq;
                ws += wq;
            }
        }
        if (lane == 0 && norm_w)
            for (int q = 0; q < k; ++q) w[q] = w[q] / ws;
        return;
    }
    // wide routers: scan the logits in memory; lane q < k remembers pick q
    // (k <= 32)
    float mx = -INFINITY;
    for (int e = lane; e < n_experts; e += 32) mx = fmaxf(mx, l[e]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.f;
    for (int e = lane; e < n_experts; e += 32) sum += expf(l[e] - mx);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    int mine = -1;
    float ws = 0.f;
    for (int q = 0; q < k; ++q) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int base = 0; base < n_experts; base += 32) {   // same trip count on every lane
            const int e = base + lane;
            bool used = e >= n_experts;
            for (int r = 0; r < q; ++r) used |= (__shfl_sync(0xffffffffu, mine, r) == e);
            if (used) continue;
            const float val = l[e];
            if (route_better(val, e, bv, bi)) { bv = val; bi = e; }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi != 0x7fffffff && route_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == q) mine = bi;
        if (lane == 0) {
            const float wq = expf(bv - mx) / sum;
            ids[q] = bi;
            w[q] = wq;
            ws += wq;
        }
    }
    if (lane == 0 && norm_w)
        for (int q = 0; q < k; ++q) w[q] = w[q] / ws;
}

}  // namespace moe
