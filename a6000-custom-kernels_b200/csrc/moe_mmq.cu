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
    static constexpr int BPB = 84;       // bytes per super-block
    static constexpr int NPLANE = 1;     // int8 planes of the folded weights
    static constexpr bool MINS = true;   // has the dmin * summs term
};

// Shared-memory layout of one CTA for weight type TYPE
template <int TYPE>
struct MmqLayout {
    using Ty = MmqType<TYPE>;
    static constexpr uint32_t SLOT = (Ty::BPB + 15) / 16 * 16 + 16;     // one row's window of one super-block
    static constexpr uint32_t CTRL = 2048;
    static constexpr uint32_t PLANE = MMQ_M * 256;                       // one int8 plane of A (32 KB)
    static constexpr uint32_t MINS_OFF = Ty::NPLANE * PLANE;             // chunks (mins, zero, mins)
    static constexpr uint32_t A_BYTES = MINS_OFF + (Ty::MINS ? 3 * (MMQ_M / 8) * 128 : 0);
    static constexpr int NA = (2 * A_BYTES <= 96u * 1024u) ? 2 : 1;     // A buffers
    static constexpr int NB = 4;                                         // B-tile stages
    static constexpr uint32_t OFF_A = CTRL;
    static constexpr uint32_t OFF_B = OFF_A + NA * A_BYTES;
    static constexpr uint32_t OFF_P = (OFF_B + NB * MMQ_BT_BYTES + 127) / 128 * 128;
    static constexpr uint32_t STAGE = MMQ_M * SLOT;
    static constexpr int NP_FIT = static_cast<int>((227u * 1024u - OFF_P) / STAGE);
    static constexpr int NP = NP_FIT > 8 ? 8 : NP_FIT;                   // weight stages
    static constexpr uint32_t TOTAL = OFF_P + NP * STAGE;
    static constexpr uint32_t ACC_COLS = 256;                            // TMEM columns per accumulator set
    static_assert(NP >= 2, "at least two weight stages");
    static_assert(TOTAL <= 227u * 1024u, "shared memory budget");
    static_assert(Ty::NPLANE * MMQ_NT + (Ty::MINS ? 2 * MMQ_NT : 0) <= ACC_COLS, "TMEM columns");
    static_assert(SLOT % 16 == 0 && SLOT <= 256, "TMA box width");
};

struct MmqCtrl {   // fits MmqLayout::CTRL (static_assert in the kernel)
    uint64_t p_full[8], p_empty[8], b_full[4], b_empty[4], mma[2];
    uint32_t tmem;
    int32_t tok[3][MMQ_NT];    // entries of the CTA's last three tiles
    float da[3][MMQ_NT];       // the tokens' block scales of the last three steps
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

// AND of v over the consumer warps (named barrier 1)
__device__ __forceinline__ bool mmq_consumer_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v ? 1u : 0u), "n"(MMQ_CWARPS * 32)
        : "memory");
    return r != 0;
}

// Q2_K super-block (84 bytes at blk) of row r -> 256 folded int8 (sc * q,
// element 16 kb + i in chunk kb) and the 16 mins (m_g = sc_g >> 4) twice,
// in the K-major layout of A; the row's d and dmin.
__device__ __forceinline__ void unpack_q2K(const uint8_t *blk, uint8_t *A, int r, float &d, float &dm) {
    uint32_t sc4[4], qs[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc4[i] = ld_u32(blk + 4 * i);
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = ld_u32(blk + 16 + 4 * i);
    uint8_t *rowp = A + (r >> 3) * 128 + (r & 7) * 16;
#pragma unroll
    for (int kb = 0; kb < 16; ++kb) {
        // elements 16 kb .. 16 kb + 15: half n = kb / 8, plane = (kb % 8) / 2,
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
    const uint4 m = make_uint4((sc4[0] >> 4) & 0x0F0F0F0Fu, (sc4[1] >> 4) & 0x0F0F0F0Fu, (sc4[2] >> 4) & 0x0F0F0F0Fu,
                               (sc4[3] >> 4) & 0x0F0F0F0Fu);
    constexpr uint32_t MO = MmqLayout<T_Q2_K>::MINS_OFF;
    *reinterpret_cast<uint4 *>(rowp + MO) = m;
    *reinterpret_cast<uint4 *>(rowp + MO + 2 * (MMQ_M / 8) * 128) = m;
    d = ld_half(blk + 80);
    dm = ld_half(blk + 82);
}

template <int TYPE>
__global__ void __launch_bounds__(MMQ_THREADS, 1) moe_mmq_kernel(const __grid_constant__ MmqArgs a) {
    using Lay = MmqLayout<TYPE>;
    using Ty = MmqType<TYPE>;
    static_assert(sizeof(MmqCtrl) <= Lay::CTRL, "control block too large");
    constexpr int BPB = Ty::BPB;
    constexpr uint32_t ACS = (MMQ_M / 8) * 128;    // A: byte stride of one 16-byte K chunk over the rows
    extern __shared__ __align__(1024) uint8_t smem[];
    MmqCtrl &C = *reinterpret_cast<MmqCtrl *>(smem);
    uint8_t *A = smem + Lay::OFF_A;
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
            mbar_init(&C.p_empty[s], MMQ_CWARPS);
        }
        for (int s = 0; s < Lay::NB; ++s) {
            mbar_init(&C.b_full[s], 1);
            mbar_init(&C.b_empty[s], 1);
        }
        mbar_init(&C.mma[0], 1);
        mbar_init(&C.mma[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        // 512 TMEM columns: two accumulator sets of ACC_COLS
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&C.tmem)),
                     "r"(2 * Lay::ACC_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (Ty::MINS && tid < MMQ_M) {   // the zero chunk between the two copies of the mins
        for (int s = 0; s < Lay::NA; ++s)
            *reinterpret_cast<uint4 *>(A + s * Lay::A_BYTES + Lay::MINS_OFF + ACS + (tid >> 3) * 128 + (tid & 7) * 16) =
                make_uint4(0, 0, 0, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = C.tmem;

    if (warp == MMQ_CWARPS) {
        // ---------------- producer warp: B tiles and weight rows -----------------
        const uint64_t pol_w = l2_evict_first_policy(), pol_b = l2_evict_last_policy();
        uint32_t ps = 0, pph = 0, bs = 0, bph = 0, fills_p = 0, fills_b = 0;
        bool pok = true;
        for (int ti = blockIdx.x; ti < total && pok; ti += gridDim.x) {
            const MmqTile T = mmq_tile(a, ti, row_blocks);
            const uint32_t bbytes = mmq_bt_bytes(mmq_chunk_n(T.nt));
            const int y0 = (T.e * a.nrows + T.rb * MMQ_M) / G;   // first tensor-map row of the tile
            for (int sb = 0; sb < nsb; ++sb) {
                bool w = lane == 0 ? mbar_wait_bounded(&C.b_empty[bs], bph ^ 1u, a.timeout_ns) : true;
                if (!__shfl_sync(0xffffffffu, w, 0)) { pok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&C.b_full[bs], bbytes);
                    bulk_g2s(B + bs * MMQ_BT_BYTES, a.btiles + (static_cast<size_t>(T.gchunk) * nsb + sb) * MMQ_BT_BYTES,
                             bbytes, &C.b_full[bs], pol_b);
                }
                ++fills_b;
                if (++bs == Lay::NB) { bs = 0; bph ^= 1u; }

                w = lane == 0 ? mbar_wait_bounded(&C.p_empty[ps], pph ^ 1u, a.timeout_ns) : true;
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
            if (!pok) set_error(a.err, DERR_TIMEOUT_EMPTY);
            // copies still in flight (only after an error): wait for every
            // stage's last fill before the block may exit
            for (uint32_t s = 0; s < static_cast<uint32_t>(Lay::NP) && s < fills_p; ++s)
                mbar_wait_bounded(&C.p_full[s], ((fills_p - 1 - s) / Lay::NP) & 1u, a.timeout_ns);
            for (uint32_t s = 0; s < static_cast<uint32_t>(Lay::NB) && s < fills_b; ++s)
                mbar_wait_bounded(&C.b_full[s], ((fills_b - 1 - s) / Lay::NB) & 1u, a.timeout_ns);
        }
    } else {
        // ---------------- consumer warps: thread r owns weight row r ---------------
        const int r = tid;
        // row r's window in a weight stage: box r % G, line r / G
        const uint32_t slot_off = static_cast<uint32_t>((r % G) * GR + r / G) * Lay::SLOT;
        const uint32_t row_in_group = static_cast<uint32_t>(r % G) * a.row_bytes;
        float acc[MMQ_NT];
#pragma unroll
        for (int n = 0; n < MMQ_NT; ++n) acc[n] = 0.f;
        uint32_t ps = 0, pph = 0, bs = 0, bph = 0, g = 0;
        float pd = 0.f, pdm = 0.f;                      // row scales of step g - 1
        int p_nt = 0, p_tb = 0, p_row = 0;              // its tile
        bool p_last = false, ok = true, mok = true;   // mok: last epilogue's MMA wait succeeded

        // finish step q (accumulator set q & 1): llama.cpp's
        // sumf += (d_a d) * isum - (d_a dmin) * summs, per token
        auto epilogue = [&](uint32_t q) {
            const uint32_t cols = tmem + (static_cast<uint32_t>(32 * warp) << 16) + (q & 1u) * Lay::ACC_COLS;
            const float *dav = C.da[q % 3];
#pragma unroll
            for (int sl = 0; sl < MMQ_NT / 16; ++sl) {
                if (sl * 16 < p_nt) {
                    uint32_t S[16], H[16], L[16];
                    tmem_ld16(cols + sl * 16, S);
                    tmem_ld16(cols + MMQ_NT + sl * 16, H);
                    tmem_ld16(cols + 2 * MMQ_NT + sl * 16, L);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float da = dav[sl * 16 + j];
                        const float dall = __fmul_rn(da, pd), dmin = __fmul_rn(da, pdm);
                        const float fi = small_int_to_float(static_cast<int>(S[j]));
                        const float fm = small_int_to_float(16 * static_cast<int>(H[j]) + static_cast<int>(L[j]));
                        acc[sl * 16 + j] = __fadd_rn(acc[sl * 16 + j], __fsub_rn(__fmul_rn(dall, fi), __fmul_rn(dmin, fm)));
                    }
                }
            }
        };
        auto store = [&]() {
            const int32_t *tk = C.tok[p_tb];
#pragma unroll
            for (int n = 0; n < MMQ_NT; ++n) {
                if (n < p_nt) a.dst[static_cast<int64_t>(tk[n]) * a.nrows + p_row] = acc[n];
                acc[n] = 0.f;
            }
        };

        int tcount = 0;
        for (int ti = blockIdx.x; ti < total && ok; ti += gridDim.x, ++tcount) {
            const MmqTile T = mmq_tile(a, ti, row_blocks);
            const int tb = tcount % 3;
            const int N = mmq_chunk_n(T.nt);
            if (tid < MMQ_NT) C.tok[tb][tid] = tid < T.nt ? a.entries[T.ebeg + T.chunk * MMQ_NT + tid] : -1;
            for (int sb = 0; sb < nsb; ++sb) {
                uint8_t *Ab = A + (g % Lay::NA) * Lay::A_BYTES;
                bool w = mok && mbar_wait_sleep(&C.p_full[ps], pph, a.timeout_ns);
                // A buffer g % NA was last read by step g - NA (waited for in
                // step g - NA + 1's epilogue when NA == 2)
                if (Lay::NA == 1 && g > 0) w &= mbar_wait_sleep(&C.mma[(g - 1) & 1u], ((g - 1) >> 1) & 1u, a.timeout_ns);
                // ---- A: this thread's row of super-block sb
                const uint8_t *slot = P + ps * Lay::STAGE + slot_off + ((row_in_group + static_cast<uint32_t>(sb) * BPB) & 15u);
                float d, dm;
                unpack_q2K(slot, Ab, r, d, dm);
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.p_empty[ps]);
                if (++ps == Lay::NP) { ps = 0; pph ^= 1u; }
                // ---- B: the chunk's tile of super-block sb
                w &= mbar_wait_sleep(&C.b_full[bs], bph, a.timeout_ns);
                const uint8_t *Bst = B + bs * MMQ_BT_BYTES;
                if (tid < MMQ_NT) C.da[g % 3][tid] = reinterpret_cast<const float *>(Bst)[tid];
                if (!w) set_error(a.err, DERR_TIMEOUT_FULL);
                fence_proxy_async_smem();
                tc_fence_before();
                ok = mmq_consumer_and(w);
                if (!ok) break;
                // ---- one thread issues the step's MMAs into accumulator set g & 1
                if (tid == 0) {
                    tc_fence_after();
                    const uint32_t bcs = 16u * N;   // B: byte stride of one 16-byte K chunk over the N tokens
                    const uint32_t idesc = umma_idesc_i8(MMQ_M, N);
                    const uint32_t a0 = smem_u32(Ab), b0 = smem_u32(Bst) + MMQ_BT_HEAD;
                    const uint32_t d0 = tmem + (g & 1u) * Lay::ACC_COLS;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        umma_i8(d0, umma_desc(a0 + kk * 2 * ACS, ACS, 128), umma_desc(b0 + kk * 2 * bcs, bcs, 128), idesc,
                                kk > 0 ? 1u : 0u);
                    if (Ty::MINS) {
                        // H = sum_g m_g hi_g (A chunks mins, zero) and L = sum_g m_g lo_g (zero, mins)
                        const uint64_t bd = umma_desc(b0 + 16 * bcs, bcs, 128);
                        umma_i8(d0 + MMQ_NT, umma_desc(a0 + Lay::MINS_OFF, ACS, 128), bd, idesc, 0u);
                        umma_i8(d0 + 2 * MMQ_NT, umma_desc(a0 + Lay::MINS_OFF + ACS, ACS, 128), bd, idesc, 0u);
                    }
                    umma_commit(&C.mma[g & 1u]);
                    umma_commit(&C.b_empty[bs]);
                }
                if (++bs == Lay::NB) { bs = 0; bph ^= 1u; }
                // ---- finish step g - 1 while this one multiplies
                if (g > 0) {
                    if (Lay::NA == 2) mok = mbar_wait_sleep(&C.mma[(g - 1) & 1u], ((g - 1) >> 1) & 1u, a.timeout_ns);
                    if (!mok) set_error(a.err, DERR_TIMEOUT_FULL);   // agreed on at the next step's barrier
                    tc_fence_after();
                    epilogue(g - 1);
                    if (p_last) store();
                    tc_fence_before();
                }
                pd = d;
                pdm = dm;
                p_nt = T.nt;
                p_tb = tb;
                p_row = T.rb * MMQ_M + r;
                p_last = sb == nsb - 1;
                ++g;
            }
        }
        if (g > 0) {
            // the last step (also waited for after an error, before TMEM is freed)
            const bool w = mbar_wait_sleep(&C.mma[(g - 1) & 1u], ((g - 1) >> 1) & 1u, a.timeout_ns);
            if (!w) set_error(a.err, DERR_TIMEOUT_FULL);
            if (ok && mok && w) {
                tc_fence_after();
                epilogue(g - 1);
                store();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * Lay::ACC_COLS)
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
    kern<<<n_sm, MMQ_THREADS, Lay::TOTAL, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { *cuda_err = e; *why = "moe_mmq_kernel launch"; return -3; }
    return 0;
}

}  // namespace moe
