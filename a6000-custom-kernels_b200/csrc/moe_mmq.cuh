// moe_mmq.cuh -- prefill MUL_MAT_ID on the 5th-generation tensor cores.
//
// With many tokens per layer (prefill), each expert is shared by several
// tokens, so its rows become a real int8 GEMM. llama.cpp runs this case as
// MMQ (the reference only claims the op: patches/apply_patches.py:81-87).
// Here:
//   * the (token, pick) entries are grouped by expert on the device; an
//     expert's entries form chunks of up to MMQ_NT tokens, and a tile is
//     (expert, 128 weight rows, one chunk);
//   * the chunks' activations are gathered once into B tiles: per chunk and
//     256-element super-block, the tokens' Q8_K quants already in the MMA's
//     shared-memory layout, plus the bsum bytes and the block scales;
//   * one CTA per SM, persistent over the tile list: a producer warp streams
//     each super-block's packed weight rows (2-D TMA boxes over groups of G
//     rows, G * row_bytes a multiple of 16) and the matching B tile into
//     shared-memory rings; four consumer warps (thread r
//     owns weight row r) unpack the row into int8 with the group scale folded
//     in (Q2_K: sc * q <= 45), so one K = 256 integer dot is exactly
//     llama.cpp's isum; the mins term summs = sum_g m_g bsum_g runs on the
//     tensor core too (bsum = 16 hi + lo, two K = 32 MMAs against the mins);
//   * one thread issues tcgen05.mma (kind::i8, M = 128, N = MMQ_NT) into one
//     of two TMEM accumulator sets, so super-block s multiplies while the
//     warps finish s - 1 with llama.cpp's float steps (vec_dot_q2_K_q8_K:
//     sumf += d_a d * isum - d_a dmin * summs), bit for bit.
#pragma once
#include <cuda.h>

#include "moe_common.cuh"

namespace moe {

constexpr int MMQ_M = 128;                 // weight rows per tile (TMEM lanes)
constexpr int MMQ_NT = 64;                 // tokens per chunk (MMA N)
constexpr int MMQ_NT32 = 16;               // tokens per chunk for the 32-weight-block types
constexpr int MMQ_CWARPS = 4;              // consumer warps: thread r owns row r
constexpr int MMQ_THREADS = 32 * (MMQ_CWARPS + 1);
constexpr int MMQ_BCHUNKS = 18;            // 16 chunks of quants + bsum hi + bsum lo (16 bytes per token each)
// B-tile head: the tokens' block scales (float [MMQ_NT]), then their 32-value
// bsum pairs (int16 [MMQ_NT][8])
constexpr uint32_t MMQ_BT_BS2 = MMQ_NT * 4;
constexpr uint32_t MMQ_BT_HEAD = MMQ_BT_BS2 + MMQ_NT * 16;
constexpr uint32_t MMQ_BT_BYTES = MMQ_BT_HEAD + MMQ_BCHUNKS * MMQ_NT * 16;
// B tile of a chunk of nt tokens: N = nt rounded up to 16 token columns
__host__ __device__ constexpr int mmq_chunk_n(int nt) { return (nt + 15) / 16 * 16; }
__host__ __device__ constexpr uint32_t mmq_bt_bytes(int n) { return MMQ_BT_HEAD + MMQ_BCHUNKS * 16u * n; }
// B tile of the 32-weight-block types (Q8_0 activations), step of sk values:
// the tokens' block scales (float [MMQ_NT32][8]), then sk / 16 quant chunks
constexpr uint32_t MMQ_BT32_HEAD = MMQ_NT32 * 8 * 4;
__host__ __device__ constexpr uint32_t mmq_bt32_bytes(int n, int sk) { return MMQ_BT32_HEAD + (sk / 16) * 16u * n; }

struct MmqArgs {
    CUtensorMap rows;               // uint8 [E * nrows / G][G * row_bytes], box {SLOT, 128 / G}
    int32_t G;                      // weight rows per tensor-map row
    const char *dense;              // expert e at dense + e * expert_bytes
    uint64_t expert_bytes;
    int32_t n_experts, K, nrows;    // per expert: nrows rows of K values
    uint32_t row_bytes;
    const uint8_t *btiles;          // [chunk][K / step][bt_stride], the first mmq_bt_bytes(N) (or _bt32_) used
    uint32_t bt_stride;             // bytes between consecutive B tiles
    int32_t n_tok, k;
    const int32_t *entries;         // entry = tok * k + pick, grouped by expert
    const int4 *chunks;             // [chunk] {expert, first entry, token count, -}; tile t is chunk t / (nrows / M)
    const int32_t *n_chunks;        // device count of chunks (chunks of up to MmqType::NT tokens)
    float *dst;                     // [tok][pick][nrows]
    int *err;
    uint64_t timeout_ns;
};

// Bound on the number of chunks of up to nt of n entries over E experts
// (workspace sizing)
__host__ __device__ constexpr int64_t mmq_max_chunks(int64_t n, int64_t E, int64_t nt) {
    return n / nt + (E < n ? E : n);
}

// ---- tcgen05 / UMMA helpers -------------------------------------------------

// Shared-memory matrix descriptor, K-major without swizzle (canonical layout:
// 8-row x 16-byte core matrices; lbo = byte distance between the two 16-byte
// K halves of a K = 32 slice, sbo = between consecutive 8-row groups).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;    // descriptor version 1 (sm_100)
    // base offset 0, leading-offset mode 0, layout type 0 (no swizzle)
    return d;
}

// Instruction descriptor of kind::i8: s32 accumulator, signed int8 A and B,
// both K-major, N x M.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (+)= A x B with A (M x 32 int8, row i in TMEM lane i, 4 elements per
// 32-bit column) in tensor memory at a_tmem and B in shared memory
__device__ __forceinline__ void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 / 16 / 8 consecutive 32-bit TMEM columns of this thread's lane (no wait)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
          "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
          "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2-D tiled TMA load of box (x, y) of `map` (x: bytes, 16-byte aligned)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane (no wait)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Exact int32 -> float for |x| < 2^22 without the conversion unit: the
// integer added to the bit pattern of 1.5 * 2^23 lands in the mantissa, and
// subtracting 1.5 * 2^23 again is exact.
__device__ __forceinline__ float small_int_to_float(int x) {
    return __fsub_rn(__int_as_float(0x4B400000 + x), 12582912.0f);
}

}  // namespace moe
