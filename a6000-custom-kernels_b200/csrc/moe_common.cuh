// moe_common.cuh -- device helpers shared by the sm_100a kernels of the MoE
// expert path: block-format constants, PTX wrappers (mbarrier, 1-D bulk copy,
// mixed-sign dp4a/dp2a), and bounded waits.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace moe {

// ggml_type ids of the path
enum : int {
    T_F32 = 0, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q8_1 = 9,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_Q8_K = 15,
};

// activation semantics
enum : int { ACT_Q8_1 = 0, ACT_CPU = 1 };

// device error codes (first writer wins)
enum : int {
    DERR_NONE = 0, DERR_BAD_ID = 1, DERR_TOO_MANY_KEYS = 2, DERR_TIMEOUT_FULL = 3,
    DERR_TIMEOUT_EMPTY = 4, DERR_TOO_MANY_SEGMENTS = 5, DERR_DRAIN = 6, DERR_GRID_BARRIER = 7,
    DERR_TIMEOUT_TAG = 8, DERR_EP_OVERFLOW = 9,
};

template <int T> struct fmt;
template <> struct fmt<T_Q4_0> { static constexpr int qk = 32,  bytes = 18,  tasks = 1; static constexpr bool a4 = false; };
template <> struct fmt<T_Q5_0> { static constexpr int qk = 32,  bytes = 22,  tasks = 1; static constexpr bool a4 = false; };
template <> struct fmt<T_Q8_0> { static constexpr int qk = 32,  bytes = 34,  tasks = 1; static constexpr bool a4 = false; };
template <> struct fmt<T_Q2_K> { static constexpr int qk = 256, bytes = 84,  tasks = 2; static constexpr bool a4 = true;  };
template <> struct fmt<T_Q3_K> { static constexpr int qk = 256, bytes = 110, tasks = 2; static constexpr bool a4 = false; };
template <> struct fmt<T_Q4_K> { static constexpr int qk = 256, bytes = 144, tasks = 4; static constexpr bool a4 = true;  };
template <> struct fmt<T_Q5_K> { static constexpr int qk = 256, bytes = 176, tasks = 4; static constexpr bool a4 = true;  };
template <> struct fmt<T_Q6_K> { static constexpr int qk = 256, bytes = 210, tasks = 2; static constexpr bool a4 = false; };

__host__ __device__ constexpr bool is_kquant(int t) { return t >= T_Q2_K && t <= T_Q6_K; }

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes or about hint_ns pass, instead of spinning on the issue slots
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Time limits are counted in SM clock cycles (clock64), taking 2 cycles per
// nanosecond: %globaltimer was seen advancing far slower than real time on
// this hardware, so it cannot bound a wait.
__device__ __forceinline__ uint64_t timeout_cycles(uint64_t timeout_ns) { return 2ull * timeout_ns; }

// Non-blocking probe of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Sleeping wait (for consumers): gives up after ~timeout_ns. Limits below
// 20 us poll with the non-blocking probe (try_wait itself may suspend for a
// hardware-defined time), so a tiny limit gives up at once.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
    if (mbar_test_wait(bar, parity)) return true;   // the common case: the phase is already complete
    if (timeout_ns < 20000u) {
        const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
        for (;;) {
            if (mbar_test_wait(bar, parity)) return true;
            if (static_cast<uint64_t>(clock64()) - t0 > lim) return false;
        }
    }
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
    const uint32_t hint = 20000u;
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, hint)) return true;
        if (static_cast<uint64_t>(clock64()) - t0 > lim) return false;
    }
}

// Limit of the wait for copies already in flight before a CTA exits: never
// below 200 ms, whatever limit the other waits run with, so a CTA whose
// other waits gave up still lets every issued copy land.
__device__ __forceinline__ uint64_t drain_limit_ns(uint64_t timeout_ns) {
    return timeout_ns > 200000000ull ? timeout_ns : 200000000ull;
}

// Wait for the phase with the given parity; gives up after ~timeout_ns.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && static_cast<uint64_t>(clock64()) - t0 > lim) return false;
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (tx bytes).
// dst, src 16-byte aligned; bytes a multiple of 16. Never used on host memory.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// sum of 4 (unsigned byte of a) * (signed byte of b) + c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// signed x signed
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// a: two signed 16-bit, b: four unsigned bytes; lo uses bytes 0,1 of b, hi bytes 2,3
__device__ __forceinline__ int dp2a_lo_su(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_su(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// a: two signed 16-bit, b: four signed bytes
__device__ __forceinline__ int dp2a_lo_ss(int a, int b, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_ss(int a, int b, int c) {
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ float ld_half(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}

// N consecutive 32-bit words from a 2-byte aligned shared-memory address
// (reads one word past the run; callers keep 16 bytes of slack).
template <int N>
__device__ __forceinline__ void ld_words_a2(const uint8_t *p, uint32_t (&w)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~static_cast<uintptr_t>(3));
    const uint32_t sh = static_cast<uint32_t>(a & 2u) * 8u;
    uint32_t x[N + 1];
#pragma unroll
    for (int i = 0; i <= N; ++i) x[i] = base[i];
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(x[i], x[i + 1], sh);
}

template <int N>
__device__ __forceinline__ void ld_words_a4(const uint8_t *p, uint32_t (&w)[N]) {
    const uint32_t *b = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = b[i];
}

// 4 bits -> bit 4 of each of the 4 bytes
__device__ __forceinline__ uint32_t spread4_bit4(uint32_t nib) { return ((nib & 0xFu) * 0x02040810u) & 0x10101010u; }

// ggml's nearest_int (1.5*2^23 magic rounding), with explicit non-contracted ops
__device__ __forceinline__ int nearest_int_dev(float prod) {
    const float val = __fadd_rn(prod, 12582912.f);
    return (__float_as_int(val) & 0x007fffff) - 0x00400000;
}

// One Q8_K block (256 values at xr) by one warp, llama.cpp's
// quantize_row_q8_K_ref: lane l quantizes values 8 l .. 8 l + 7 into q
// (scale -127 / (the value of largest magnitude, first index on ties), values
// clamped to 127); returns d = 1 / iscale (0 for an all-zero block) and in s
// the lane's 8-value sum plus its neighbour's (lane 2 g then holds bsum g).
// (quant_q8K_vals: the same from the lane's 8 values already loaded)
__device__ __forceinline__ float quant_q8K_vals(const float (&v)[8], int lane, int8_t (&q)[8], int &s) {
    float amax = 0.f, mval = 0.f;
    int midx = 1 << 30;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
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
    s = 0;
    float d = 0.f;
    if (amax != 0.f) {
        const float iscale = -127.f / mval;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = nearest_int_dev(__fmul_rn(iscale, v[j]));
            q[j] = static_cast<int8_t>(r < 127 ? r : 127);
            s += q[j];
        }
        d = 1.f / iscale;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = 0;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    return d;
}
__device__ __forceinline__ float quant_q8K_warp(const float *__restrict__ xr, int lane, int8_t (&q)[8], int &s) {
    const float4 a = *reinterpret_cast<const float4 *>(xr + lane * 8);
    const float4 b = *reinterpret_cast<const float4 *>(xr + lane * 8 + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    return quant_q8K_vals(v, lane, q, s);
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Atomic add with acquire-release semantics at GPU scope: releases what the
// caller (and, through a preceding CTA barrier, its CTA) wrote, and acquires
// what the earlier adders released. Returns the old value.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// System-scope (other GPUs) release / acquire on 32-bit words.
__device__ __forceinline__ void red_release_sys_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// two 64-bit words at a 16-byte aligned address (each word single-copy atomic)
__device__ __forceinline__ void ld_relaxed_u64x2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// GLU epilogue (reference kernels/moe-cache.cu:264-280): result = up, g = gate
__device__ __forceinline__ float glu_apply(int op, float g, float up, float limit) {
    switch (op) {
        case 0: return up * (g / (1.0f + expf(-g)));
        case 1: {
            const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
            return up * (0.5f * g * (1.0f + tanhf(c * g * (1.0f + a * g * g))));
        }
        case 2: {
            const float x = fminf(g, 7.0f);
            const float u = fmaxf(fminf(up, 7.0f), -7.0f);
            return (x / (1.0f + expf(-x * 1.702f))) * (u + 1.0f);
        }
        case 3: {
            const float x = fminf(g, limit);
            const float u = fmaxf(fminf(up, limit), -limit);
            return (x / (1.0f + expf(-x))) * u;
        }
        default: return up * g;
    }
}

}  // namespace moe
