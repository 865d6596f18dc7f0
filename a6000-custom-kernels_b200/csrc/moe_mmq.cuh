// moe_mmq.cuh -- prefill MUL_MAT_ID on the 5th-generation tensor cores.
//
// With many tokens per layer (prefill), each expert is shared by several
// tokens, so its rows become a real int8 GEMM. llama.cpp runs this case as
// MMQ (the reference only claims the op: patches/apply_patches.py:81-87).
// Here:
//   * tokens are grouped by expert on the device (counts, offsets, entries);
//   * a tile is (expert, 128 weight rows, up to MMQ_NT tokens); one CTA of 4
//     warps per tile, persistent over the tile list;
//   * the tile's packed rows arrive by one bulk copy; per 256-element
//     super-block the warps unpack them into int8 operands in shared memory
//     with the 16-element group scale folded in (Q2_K: sc * q <= 45; Q3_K:
//     sc * q in [-128, 124]), so one K = 256 integer dot per (row, token) is
//     exactly llama.cpp's isum; the activations are the tokens' Q8_K blocks;
//   * one thread issues tcgen05.mma (kind::i8, M = 128, N = MMQ_NT, 8 x
//     K = 32) into one of two TMEM accumulators, so the next super-block is
//     unpacked while the tensor core works;
//   * the warps read the int32 sums back (tcgen05.ld) and finish each
//     super-block with llama.cpp's float arithmetic (vec_dot_q2_K_q8_K:
//     sumf += d_a d * isum - d_a dmin * summs), so results match the CPU
//     path bit for bit.
#pragma once
#include "moe_common.cuh"

namespace moe {

constexpr int MMQ_M = 128;          // weight rows per tile (TMEM lanes)
constexpr int MMQ_NT = 32;          // tokens per tile (MMA N)
constexpr int MMQ_THREADS = 128;    // 4 warps: thread r owns row r of the tile
constexpr int MMQ_MAX_PACKED = 128 * 1008;   // packed rows of one tile in shared memory (Q2_K, K = 3072)

struct MmqArgs {
    const char *const *tbl;         // expert table (tagged pointers) or null
    const char *dense;              // expert e at dense + e * expert_bytes when tbl is null
    uint64_t expert_bytes;
    int32_t n_experts, K, nrows;    // per expert: nrows rows of K values
    uint32_t row_bytes;
    const uint8_t *x8;              // Q8_K activations [n_tok][K / 256] blocks of 292 bytes
    int32_t n_tok, k;
    const int32_t *offsets;         // [n_experts + 1] into entries
    const int32_t *entries;         // entry = tok * k + pick, grouped by expert
    const int32_t *tile_off;        // [n_experts + 1] tile prefix; tiles of e: ceil(cnt / NT) x (nrows / M)
    float *dst;                     // [tok][pick][nrows]
    int *err;
    uint64_t timeout_ns;
};

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

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive 32-bit TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace moe
