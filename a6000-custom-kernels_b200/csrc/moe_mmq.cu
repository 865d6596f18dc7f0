// moe_mmq.cu -- prefill MUL_MAT_ID on tcgen05 (see moe_mmq.cuh): grouping of
// (token, pick) entries by expert and the grouped int8 GEMM.
#include <cstdio>

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
// The grouped GEMM
// ---------------------------------------------------------------------------
template <int TYPE>
struct mmq_fmt;
template <> struct mmq_fmt<T_Q2_K> { static constexpr int bytes = 84; };

// Shared-memory layout of one CTA
struct MmqSmem {
    static constexpr uint32_t A_BYTES = MMQ_M * 256;          // one super-block of int8 A (32 KB)
    static constexpr uint32_t B_BYTES = MMQ_NT * 256;         // one super-block of int8 B (8 KB)
    static constexpr uint32_t CTRL = 4096;
    static constexpr uint32_t OFF_A = CTRL;
    static constexpr uint32_t OFF_B = OFF_A + 2 * A_BYTES;
    static constexpr uint32_t OFF_P = OFF_B + 2 * B_BYTES;    // packed rows
    static constexpr uint32_t TOTAL = OFF_P + MMQ_MAX_PACKED;
};

struct MmqCtrl {   // fits MmqSmem::CTRL (static_assert below)
    uint64_t bar_p, bar_mma[2];
    uint32_t tmem;
    int32_t tok_entry[MMQ_NT];
    float da[2][MMQ_NT];
    int16_t bsum[2][MMQ_NT][16];
};

static_assert(sizeof(MmqCtrl) <= MmqSmem::CTRL, "control block too large");
static_assert(MmqSmem::TOTAL <= 227 * 1024, "shared memory budget");

// Q2_K super-block sb of one row (84 bytes at blk) -> 256 folded int8
// (sc * q) in the K-major canonical layout at A + row offset
__device__ __forceinline__ void unpack_q2K(const uint8_t *blk, uint8_t *A, int r) {
    uint32_t sc4[4], qs[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc4[i] = ld_u32(blk + 4 * i);
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = ld_u32(blk + 16 + 4 * i);
    uint8_t *rowp = A + (r >> 3) * 128 + (r & 7) * 16;
#pragma unroll
    for (int kb = 0; kb < 16; ++kb) {
        // 16 elements 16 kb .. 16 kb + 15: half n = kb / 8, plane = (kb % 8) / 2,
        // bytes 16 (kb % 2) .. + 15 of the half's 32 quant bytes; one scale
        const int n = kb >> 3, plane = (kb & 7) >> 1, hb = kb & 1;
        const uint32_t sc = (sc4[kb >> 2] >> (8 * (kb & 3))) & 0xFu;
        uint4 v;
        v.x = ((qs[8 * n + 4 * hb + 0] >> (2 * plane)) & 0x03030303u) * sc;
        v.y = ((qs[8 * n + 4 * hb + 1] >> (2 * plane)) & 0x03030303u) * sc;
        v.z = ((qs[8 * n + 4 * hb + 2] >> (2 * plane)) & 0x03030303u) * sc;
        v.w = ((qs[8 * n + 4 * hb + 3] >> (2 * plane)) & 0x03030303u) * sc;
        *reinterpret_cast<uint4 *>(rowp + kb * (MMQ_M / 8) * 128) = v;
    }
}

template <int TYPE>
__global__ void __launch_bounds__(MMQ_THREADS, 1) moe_mmq_kernel(const __grid_constant__ MmqArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    MmqCtrl &C = *reinterpret_cast<MmqCtrl *>(smem);
    uint8_t *A = smem + MmqSmem::OFF_A;
    uint8_t *B = smem + MmqSmem::OFF_B;
    uint8_t *P = smem + MmqSmem::OFF_P;
    const int tid = threadIdx.x, warp = tid >> 5;
    constexpr int BPB = mmq_fmt<TYPE>::bytes;
    const int nsb = a.K / 256;
    const int row_blocks = a.nrows / MMQ_M;
    constexpr uint32_t IDESC = umma_idesc_i8(MMQ_M, MMQ_NT);

    if (tid == 0) {
        mbar_init(&C.bar_p, 1);
        mbar_init(&C.bar_mma[0], 1);
        mbar_init(&C.bar_mma[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        // 64 TMEM columns: two accumulators of MMQ_NT int32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&C.tmem)),
                     "r"(64u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = C.tmem;
    uint32_t ph_p = 0, ph_mma[2] = {0, 0};
    bool ok = true;
    const int total = a.tile_off[a.n_experts];

    for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x) {
        // tile -> expert (binary search of the tile prefix), row block, token chunk
        int lo = 0, hi = a.n_experts;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (a.tile_off[mid] <= ti) lo = mid;
            else hi = mid;
        }
        const int e = lo;
        const int local = ti - a.tile_off[e];
        const int rb = local % row_blocks, chunk = local / row_blocks;
        const int ebeg = a.offsets[e], ecnt = a.offsets[e + 1] - ebeg;
        const int nt = min(MMQ_NT, ecnt - chunk * MMQ_NT);
        if (tid < MMQ_NT) C.tok_entry[tid] = tid < nt ? a.entries[ebeg + chunk * MMQ_NT + tid] : -1;
        // packed rows of the tile: one bulk copy (row block rb of expert e)
        const char *src;
        if (a.tbl) src = reinterpret_cast<const char *>(reinterpret_cast<uintptr_t>(a.tbl[e]) & ~static_cast<uintptr_t>(1));
        else src = a.dense + static_cast<uint64_t>(e) * a.expert_bytes;
        src += static_cast<uint64_t>(rb) * MMQ_M * a.row_bytes;
        const uint32_t pbytes = MMQ_M * a.row_bytes;
        if (tid == 0) {
            mbar_arrive_expect_tx(&C.bar_p, pbytes);
            for (uint32_t off = 0; off < pbytes; off += 32768u) {
                const uint32_t n = pbytes - off < 32768u ? pbytes - off : 32768u;
                bulk_g2s(P + off, src + off, n, &C.bar_p, l2_evict_first_policy());
            }
        }
        __syncthreads();
        if (!mbar_wait_sleep(&C.bar_p, ph_p, a.timeout_ns)) {
            if (tid == 0) set_error(a.err, DERR_TIMEOUT_FULL);
            ok = false;
        }
        ph_p ^= 1u;
        ok = __syncthreads_and(ok);   // every thread leaves together
        if (!ok) break;

        float acc[MMQ_NT];
#pragma unroll
        for (int n = 0; n < MMQ_NT; ++n) acc[n] = 0.f;
        float dw[2] = {0.f, 0.f}, dmw[2] = {0.f, 0.f};
        uint32_t mins[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
        const uint8_t *prow = P + static_cast<size_t>(tid) * a.row_bytes;

        // finish super-block s (accumulator / buffers b): llama.cpp's
        // sumf += d_a d * isum - d_a dmin * summs
        auto epilogue = [&](int b) {
            uint32_t S[32];
            tc_fence_after();
            tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(b * MMQ_NT), S);
#pragma unroll
            for (int n = 0; n < MMQ_NT; ++n) {
                int summs = 0;
#pragma unroll
                for (int g = 0; g < 16; ++g)
                    summs += static_cast<int>(C.bsum[b][n][g]) * static_cast<int>((mins[b][g >> 2] >> (8 * (g & 3))) & 0xFu);
                const float da = C.da[b][n];
                const float dall = __fmul_rn(da, dw[b]), dmin = __fmul_rn(da, dmw[b]);
                const float t = __fsub_rn(__fmul_rn(dall, static_cast<float>(static_cast<int>(S[n]))),
                                          __fmul_rn(dmin, static_cast<float>(summs)));
                acc[n] = __fadd_rn(acc[n], t);
            }
            tc_fence_before();
        };

        for (int sb = 0; sb < nsb; ++sb) {
            const int b = sb & 1;
            // ---- A: this thread's row, super-block sb, folded int8
            const uint8_t *blk = prow + static_cast<size_t>(sb) * BPB;
            unpack_q2K(blk, A + b * MmqSmem::A_BYTES, tid);
            dw[b] = ld_half(blk + 80);
            dmw[b] = ld_half(blk + 82);
#pragma unroll
            for (int i = 0; i < 4; ++i) mins[b][i] = (ld_u32(blk + 4 * i) >> 4) & 0x0F0F0F0Fu;
            // ---- B: the tokens' Q8_K quants of super-block sb (4 threads per token)
            {
                const int n = tid >> 2, part = tid & 3;     // 64 bytes each
                const int ent = C.tok_entry[n];
                uint8_t *bb = B + b * MmqSmem::B_BYTES + (n >> 3) * 128 + (n & 7) * 16;
                if (ent >= 0) {
                    const uint8_t *q8 = a.x8 + (static_cast<size_t>(ent / a.k) * nsb + sb) * 292;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int kb = part * 4 + c;
                        uint4 v;
                        v.x = __ldg(reinterpret_cast<const uint32_t *>(q8 + 4 + 16 * kb));
                        v.y = __ldg(reinterpret_cast<const uint32_t *>(q8 + 8 + 16 * kb));
                        v.z = __ldg(reinterpret_cast<const uint32_t *>(q8 + 12 + 16 * kb));
                        v.w = __ldg(reinterpret_cast<const uint32_t *>(q8 + 16 + 16 * kb));
                        *reinterpret_cast<uint4 *>(bb + kb * (MMQ_NT / 8) * 128) = v;
                    }
                    if (part == 0) C.da[b][n] = __ldg(reinterpret_cast<const float *>(q8));
                    if (part < 2) {
#pragma unroll
                        for (int g = 0; g < 8; ++g)
                            C.bsum[b][n][8 * part + g] =
                                static_cast<int16_t>(__ldg(reinterpret_cast<const unsigned short *>(q8 + 260) + 8 * part + g));
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4 *>(bb + (part * 4 + c) * (MMQ_NT / 8) * 128) = make_uint4(0, 0, 0, 0);
                    if (part == 0) C.da[b][n] = 0.f;
                    if (part < 2)
#pragma unroll
                        for (int g = 0; g < 8; ++g) C.bsum[b][n][8 * part + g] = 0;
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            // ---- one thread: 8 MMAs of K = 32 into accumulator b
            if (tid == 0) {
                tc_fence_after();
                const uint32_t a0 = smem_u32(A + b * MmqSmem::A_BYTES), b0 = smem_u32(B + b * MmqSmem::B_BYTES);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t da_ = umma_desc(a0 + kk * 2 * (MMQ_M / 8) * 128, (MMQ_M / 8) * 128, 128);
                    const uint64_t db_ = umma_desc(b0 + kk * 2 * (MMQ_NT / 8) * 128, (MMQ_NT / 8) * 128, 128);
                    umma_i8(tmem + static_cast<uint32_t>(b * MMQ_NT), da_, db_, IDESC, kk > 0 ? 1u : 0u);
                }
                umma_commit(&C.bar_mma[b]);
            }
            // ---- finish the previous super-block while this one multiplies
            if (sb > 0) {
                const int pb = b ^ 1;
                if (!mbar_wait_sleep(&C.bar_mma[pb], ph_mma[pb], a.timeout_ns)) {
                    if (tid == 0) set_error(a.err, DERR_TIMEOUT_FULL);
                    ok = false;
                }
                ph_mma[pb] ^= 1u;
                epilogue(pb);
            }
            ok = __syncthreads_and(ok);   // buffers of super-block sb - 1 are free again
            if (!ok) break;
        }
        if (!ok) break;
        {
            const int lb = (nsb - 1) & 1;
            if (!mbar_wait_sleep(&C.bar_mma[lb], ph_mma[lb], a.timeout_ns)) {
                if (tid == 0) set_error(a.err, DERR_TIMEOUT_FULL);
                ok = false;
            }
            ph_mma[lb] ^= 1u;
            epilogue(lb);
        }
        // ---- outputs: row rb * M + tid for each token of the tile
        const int row = rb * MMQ_M + tid;
#pragma unroll
        for (int n = 0; n < MMQ_NT; ++n) {
            const int ent = C.tok_entry[n];
            if (ent >= 0) a.dst[static_cast<int64_t>(ent) * a.nrows + row] = acc[n];
        }
        __syncthreads();   // packed rows and token list are free for the next tile
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64u) : "memory");
}

cudaError_t launch_mmq_group(const int32_t *ids, int64_t ids_stride, int n_tok, int k, int E, int row_blocks,
                             int32_t *cnt, int32_t *offsets, int32_t *cursor, int32_t *entries, int32_t *tile_off,
                             int *err, cudaStream_t st) {
    mmq_group_kernel<<<1, 1024, 0, st>>>(ids, ids_stride, n_tok, k, E, row_blocks, cnt, offsets, cursor, entries,
                                         tile_off, err);
    return cudaGetLastError();
}

int launch_mmq(int type, MmqArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err) {
    *cuda_err = cudaSuccess;
    if (type != T_Q2_K) { *why = "tensor-core prefill handles Q2_K"; return -2; }
    if (a.K % 256 || a.nrows % MMQ_M) { *why = "prefill MMQ needs K % 256 == 0 and rows % 128 == 0"; return -2; }
    if (static_cast<uint64_t>(MMQ_M) * a.row_bytes > MMQ_MAX_PACKED) { *why = "rows too wide for the packed tile"; return -2; }
    if (a.timeout_ns == 0) a.timeout_ns = 2000000000ull;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -3;
    auto kern = moe_mmq_kernel<T_Q2_K>;
    if (!configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MmqSmem::TOTAL);
        if (e != cudaSuccess) { *cuda_err = e; *why = "cudaFuncSetAttribute"; return -3; }
        configured[dev] = true;
    }
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    kern<<<n_sm, MMQ_THREADS, MmqSmem::TOTAL, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { *cuda_err = e; *why = "moe_mmq_kernel launch"; return -3; }
    return 0;
}

}  // namespace moe
