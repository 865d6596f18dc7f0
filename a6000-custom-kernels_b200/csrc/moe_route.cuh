// moe_route.cuh -- top-k routing of one token by one warp, shared by the
// stand-alone routing kernel and the fused layer kernel so both give the same
// bits. It restates llama.cpp's MoE gating (build_moe_ffn: softmax over the
// router logits, argsort top-k, optional renormalisation over the k picks).
#pragma once
#include <cmath>
#include <cstdint>

namespace moe {

// Order-preserving 32-bit key of a logit: larger logit -> larger key (NaN
// above +inf or below -inf by sign); -0 is folded into +0 first so that equal
// logits get equal keys. Key 0 is below every logit ("no candidate").
__device__ __forceinline__ uint32_t logit_key(float x) {
    const uint32_t u = __float_as_uint(__fadd_rn(x, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_logit(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Selection, register path for n_experts <= 32 * NV: lane l holds experts
// l + 32 j. The order is (logit descending, expert id ascending). Each pick
// reduces the lane's untaken candidates with a pairwise tree (left halves
// hold the lower ids, so the right side wins only when strictly larger),
// then the warp with redux max (key) and redux min (id among equal keys).
// Lane q < k writes ids[q].
template <int NV>
__device__ __forceinline__ void route_select_regs(const float *__restrict__ l, int n_experts, int k, int lane,
                                                  int32_t *ids) {
    uint32_t key[NV];
    uint32_t live = 0;   // bit j: expert lane + 32 j exists and is not picked yet
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int e = lane + 32 * j;
        const bool ok = e < n_experts;
        key[j] = ok ? logit_key(l[e]) : 0u;
        live |= (ok ? 1u : 0u) << j;
    }
    uint32_t pick = 0;   // lane q keeps pick q
    for (int q = 0; q < k; ++q) {
        uint32_t tk[NV];
        int tj[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) { tk[j] = ((live >> j) & 1u) ? key[j] : 0u; tj[j] = j; }
#pragma unroll
        for (int width = 1; width < NV; width *= 2) {
#pragma unroll
            for (int j = 0; j + width < NV; j += 2 * width) {
                const bool right = tk[j + width] > tk[j];
                tk[j] = right ? tk[j + width] : tk[j];
                tj[j] = right ? tj[j + width] : tj[j];
            }
        }
        const uint32_t wk = __reduce_max_sync(0xffffffffu, tk[0]);
        const uint32_t mine = (tk[0] == wk && wk != 0u) ? static_cast<uint32_t>(lane + 32 * tj[0]) : 0xFFFFFFFFu;
        const uint32_t wi = __reduce_min_sync(0xffffffffu, mine);
        if (static_cast<int>(wi & 31u) == lane) live &= ~(1u << (wi >> 5));
        if (lane == q) pick = wi;
    }
    if (lane < k) ids[lane] = static_cast<int32_t>(pick);
}

// Selection for any n_experts: scan the logits in memory; lane q < k
// remembers pick q (k <= 32) and writes ids[q].
__device__ __forceinline__ void route_select_wide(const float *__restrict__ l, int n_experts, int k, int lane,
                                                  int32_t *ids) {
    int mine = -1;
    for (int q = 0; q < k; ++q) {
        uint32_t bk = 0;
        int bi = 0x7fffffff;
        for (int base = 0; base < n_experts; base += 32) {   // same trip count on every lane
            const int e = base + lane;
            bool used = e >= n_experts;
            for (int r = 0; r < q; ++r) used |= (__shfl_sync(0xffffffffu, mine, r) == e);
            const uint32_t kv = used ? 0u : logit_key(l[e]);
            if (kv > bk) { bk = kv; bi = e; }     // ascending e: ties keep the lower id
        }
        const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
        const int wi = static_cast<int>(__reduce_min_sync(0xffffffffu, bk == wk ? static_cast<uint32_t>(bi) : 0xFFFFFFFFu));
        if (lane == q) mine = wi;
    }
    if (lane < k) ids[lane] = mine;
}

// Top-k of one token's logits l[0..n_experts) (descending, ties to the lower
// expert id; NaN logits rank by their key). Lane q < k writes ids[q]; all 32
// lanes call; k <= 32.
__device__ __forceinline__ void route_select(const float *__restrict__ l, int n_experts, int k, int lane,
                                             int32_t *ids) {
    if (n_experts <= 32 * 8) route_select_regs<8>(l, n_experts, k, lane, ids);
    else if (n_experts <= 32 * 16) route_select_regs<16>(l, n_experts, k, lane, ids);
    else route_select_wide(l, n_experts, k, lane, ids);
}

// Top-k of one warp's slice [lo, lo + 32 NV) of the logits (n_experts caps
// it): lane q < k receives pick q of the slice as (key, id), key 0 where the
// slice has fewer than q + 1 experts. Order as route_select.
template <int NV>
__device__ __forceinline__ void route_slice_topk(const float *__restrict__ l, int lo, int n_experts, int k, int lane,
                                                 uint32_t &out_key, int &out_id) {
    uint32_t key[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int e = lo + lane + 32 * j;
        key[j] = e < n_experts ? logit_key(l[e]) : 0u;
    }
    out_key = 0;
    out_id = 0x7fffffff;
    for (int q = 0; q < k; ++q) {
        uint32_t tk = 0;
        int tj = 0;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (key[j] > tk) { tk = key[j]; tj = j; }      // ascending j: ties keep the lower id
        const uint32_t wk = __reduce_max_sync(0xffffffffu, tk);
        const uint32_t mine = (tk == wk && wk != 0u) ? static_cast<uint32_t>(lo + lane + 32 * tj) : 0xFFFFFFFFu;
        const uint32_t wi = __reduce_min_sync(0xffffffffu, mine);
        if (wk != 0u && static_cast<int>((wi - lo) & 31u) == lane) {
#pragma unroll
            for (int j = 0; j < NV; ++j)
                if (static_cast<uint32_t>(lo + lane + 32 * j) == wi) key[j] = 0u;
        }
        if (lane == q) { out_key = wk; out_id = wk ? static_cast<int>(wi) : 0x7fffffff; }
    }
}

// Top-k over n_experts logits by NW warps of a block: warp w takes the slice
// [w CH, (w + 1) CH) (CH = 32 NV) and keeps its k best in cand_key/cand_id
// [w * k + q]; after the caller's barrier, merge_topk (one warp) picks the k
// best of the NW * k candidates. Every global pick is among its slice's k
// best, so the result equals route_select's bit for bit. k <= 16.
template <int NV>
__device__ __forceinline__ void route_block_slices(const float *__restrict__ l, int n_experts, int k, int warp,
                                                   int lane, uint32_t *cand_key, int *cand_id) {
    uint32_t kk;
    int id;
    route_slice_topk<NV>(l, warp * 32 * NV, n_experts, k, lane, kk, id);
    if (lane < k) { cand_key[warp * k + lane] = kk; cand_id[warp * k + lane] = id; }
}

// Rank selection without serial rounds, for n_experts <= 32 * NWARPS:
// stage 1 -- warp w holds experts 32 w + lane and ranks each within its
// warp by counting the warp's keys ahead of it (key desc, id asc; 32
// shuffles); its k best go to cand[w * k + rank]. Stage 2 (after the
// caller's barrier) -- every candidate is ranked among all NWARPS * k
// candidates by 4 threads counting 1/4 each; rank q < k is pick q.
__device__ __forceinline__ void rank_slice(const float *__restrict__ l, int n_experts, int k, int warp, int lane,
                                           uint32_t *cand_key, int *cand_id) {
    const int e = 32 * warp + lane;
    const uint32_t key = e < n_experts ? logit_key(l[e]) : 0u;
    int ahead = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const uint32_t kj = __shfl_sync(0xffffffffu, key, j);
        ahead += (kj > key || (kj == key && j < lane)) ? 1 : 0;
    }
    if (ahead < k) {
        cand_key[warp * k + ahead] = key;
        cand_id[warp * k + ahead] = e;
    }
}
// nthreads >= 4 * nc threads call with their thread index; lanes of one
// group of 4 are consecutive.
__device__ __forceinline__ void rank_candidates(const uint32_t *cand_key, const int *cand_id, int nc, int k, int tid,
                                                int32_t *ids) {
    const int c = tid >> 2, part = tid & 3;
    const bool live = c < nc;
    const uint32_t key = live ? cand_key[c] : 0u;
    const int id = live ? cand_id[c] : 0x7fffffff;
    int ahead = 0;
    for (int d = part; d < nc; d += 4) {
        const uint32_t kd = cand_key[d];
        const int idd = cand_id[d];
        ahead += (kd > key || (kd == key && idd < id)) ? 1 : 0;
    }
    ahead += __shfl_xor_sync(0xffffffffu, ahead, 1);
    ahead += __shfl_xor_sync(0xffffffffu, ahead, 2);
    if (live && part == 0 && ahead < k) ids[ahead] = id;
}

// The k best of nc <= 32 MAXC candidates (key, id), order (key desc, id
// asc); lane q < k writes ids[q]. Lane l holds candidates l + 32 j.
template <int MAXC>
__device__ __forceinline__ void merge_topk_n(const uint32_t *cand_key, const int *cand_id, int nc, int k, int lane,
                                             int32_t *ids) {
    uint32_t ck[MAXC];
    int ci[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
        const int c = lane + 32 * j;
        ck[j] = c < nc ? cand_key[c] : 0u;
        ci[j] = c < nc ? cand_id[c] : 0x7fffffff;
    }
    int pick = -1;
    for (int q = 0; q < k; ++q) {
        uint32_t bk = ck[0];
        int bi = ci[0], bj = 0;
#pragma unroll
        for (int j = 1; j < MAXC; ++j)
            if (ck[j] > bk || (ck[j] == bk && ci[j] < bi)) { bk = ck[j]; bi = ci[j]; bj = j; }
        const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
        const int wi = static_cast<int>(__reduce_min_sync(0xffffffffu, bk == wk ? static_cast<uint32_t>(bi) : 0xFFFFFFFFu));
        if (bk == wk && bi == wi) {
#pragma unroll
            for (int j = 0; j < MAXC; ++j)
                if (j == bj) ck[j] = 0u;
        }
        if (lane == q) pick = wi;
    }
    if (lane < k) ids[lane] = pick;
}
__device__ __forceinline__ void merge_topk(const uint32_t *cand_key, const int *cand_id, int nc, int k, int lane,
                                           int32_t *ids) {
    if (nc <= 32) merge_topk_n<1>(cand_key, cand_id, nc, k, lane, ids);
    else if (nc <= 64) merge_topk_n<2>(cand_key, cand_id, nc, k, lane, ids);
    else if (nc <= 128) merge_topk_n<4>(cand_key, cand_id, nc, k, lane, ids);
    else if (nc <= 256) merge_topk_n<8>(cand_key, cand_id, nc, k, lane, ids);
    else merge_topk_n<16>(cand_key, cand_id, nc, k, lane, ids);
}

// Gating weights of the picks ids[0..k) (written by this warp or visible to
// it): softmax over all experts, expf(l - max) / sum_e expf(l_e - max) with
// the sum taken lane-strided (lane j adds experts j, j + 32, ... in order) and
// then over the lanes by xor butterfly; with norm_w each weight is divided by
// the k weights' sum in pick order. Lane q < k writes w[q].
__device__ __forceinline__ void route_weights(const float *__restrict__ l, int n_experts, int k, int norm_w,
                                              int lane, const int32_t *ids, float *w) {
    uint32_t lmax = 0;
    for (int e = lane; e < n_experts; e += 32) lmax = max(lmax, logit_key(l[e]));
    const float mx = key_logit(__reduce_max_sync(0xffffffffu, lmax));
    float sum = 0.f;
    for (int e = lane; e < n_experts; e += 32) sum += expf(l[e] - mx);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float wq = lane < k ? expf(l[ids[lane]] - mx) / sum : 0.f;
    if (norm_w) {
        float ws = 0.f;
        for (int q = 0; q < k; ++q) ws += __shfl_sync(0xffffffffu, wq, q);
        if (lane < k) w[lane] = wq / ws;
    } else if (lane < k) {
        w[lane] = wq;
    }
}

// Both: the picks, then their weights.
__device__ __forceinline__ void route_token_warp(const float *__restrict__ l, int n_experts, int k, int norm_w,
                                                 int lane, int32_t *ids, float *w) {
    route_select(l, n_experts, k, lane, ids);
    __syncwarp();
    route_weights(l, n_experts, k, norm_w, lane, ids, w);
}

}  // namespace moe
