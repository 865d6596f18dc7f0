// moe_ep.cu -- expert-parallel prefill exchange over NVLink peer memory.
//
// Every GPU owns exchange buffers in its own HBM, mapped into the other GPUs
// by CUDA IPC: received rows x [W * cap][H], their local expert ids and
// source entries [W * cap] (region s = rows from GPU s, cap = that GPU's
// entries, so no count is needed before sending), the outputs of its own
// entries returned by their owners y_ret [cap][H], and two arrival counters.
// Dispatch: each GPU writes every (token, pick) entry's row and ids straight
// into the owner's region for it (peer stores, one warp per entry), marks the
// rest of each region empty (-1), and adds 1 to each owner's dispatch counter
// after a system fence. Owners wait until the counter reaches W per layer
// call, run the expert prefill on their regions (empty slots skipped),
// write each output row back into its source's y_ret, and add 1 to each
// source's return counter. No host round trip: the counters carry the sizes.
// Every wait is bounded (an error word on timeout, never a trap).
#include <cstring>

#include "moe_aux.h"
#include "moe_common.cuh"

namespace moe {

constexpr int EP_MAX_WORLD = 8;

struct EpPeers {
    float *x[EP_MAX_WORLD];
    int32_t *ids[EP_MAX_WORLD];
    int32_t *src[EP_MAX_WORLD];
    float *y_ret[EP_MAX_WORLD];
    uint32_t *flags[EP_MAX_WORLD];
};

// owner of global expert e: the last rank r with E r / W <= e (balanced
// contiguous slices)
__device__ __forceinline__ int ep_owner(int e, int E, int W) {
    int r = 0;
    for (int q = 1; q < W; ++q)
        if (static_cast<int64_t>(E) * q / W <= e) r = q;
    return r;
}

__device__ __forceinline__ void red_add_sys(uint32_t *p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Block-level "last one out" after every block's stores: returns true in the
// last block to finish (all other blocks' writes fenced before its count).
__device__ __forceinline__ bool ep_last_block(uint32_t *done) {
    __shared__ bool last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) __threadfence();
    return last;
}

__global__ void ep_dispatch_kernel(EpPeers P, int W, int me, int cap, const int32_t *__restrict__ ids, int n_entries,
                                   int k, int E, const float *__restrict__ x, int H, uint32_t *cursor, uint32_t *done,
                                   int *err) {
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n_entries; i += nwarps) {
        const int e = ids[i];
        if (e < 0 || e >= E) {
            if (lane == 0) set_error(err, DERR_BAD_ID);
            continue;
        }
        const int d = ep_owner(e, E, W);
        const int lo = static_cast<int>(static_cast<int64_t>(E) * d / W);
        uint32_t slot = 0;
        if (lane == 0) slot = atomicAdd(&cursor[d], 1u);
        slot = __shfl_sync(0xffffffffu, slot, 0);
        if (slot >= static_cast<uint32_t>(cap)) {   // more entries than the region holds: a caller error
            if (lane == 0) set_error(err, DERR_EP_OVERFLOW);
            continue;
        }
        const size_t row = static_cast<size_t>(me) * cap + slot;
        const float4 *s4 = reinterpret_cast<const float4 *>(x + static_cast<size_t>(i / k) * H);
        float4 *d4 = reinterpret_cast<float4 *>(P.x[d] + row * H);
        for (int c = lane; c < H / 4; c += 32) d4[c] = s4[c];
        if (lane == 0) {
            P.ids[d][row] = e - lo;
            P.src[d][row] = i;
        }
    }
    if (!ep_last_block(done)) return;
    // the rest of each owner's region for this GPU is empty
    for (int d = 0; d < W; ++d) {
        const uint32_t used = *reinterpret_cast<volatile uint32_t *>(&cursor[d]);
        for (uint32_t c = used + threadIdx.x; c < static_cast<uint32_t>(cap); c += blockDim.x)
            P.ids[d][static_cast<size_t>(me) * cap + c] = -1;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < static_cast<unsigned>(W)) red_add_sys(P.flags[threadIdx.x] + 0, 1u);
    __syncthreads();
    if (threadIdx.x < static_cast<unsigned>(W)) cursor[threadIdx.x] = 0;
    if (threadIdx.x == 0) *done = 0;
}

__global__ void ep_return_kernel(EpPeers P, int W, int cap, const int32_t *__restrict__ ids,
                                 const int32_t *__restrict__ src, const float *__restrict__ y, int H, uint32_t *done) {
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int rows = W * cap;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
        if (ids[r] < 0) continue;
        const int s = r / cap, entry = src[r];
        const float4 *s4 = reinterpret_cast<const float4 *>(y + static_cast<size_t>(r) * H);
        float4 *d4 = reinterpret_cast<float4 *>(P.y_ret[s] + static_cast<size_t>(entry) * H);
        for (int c = lane; c < H / 4; c += 32) d4[c] = s4[c];
    }
    if (!ep_last_block(done)) return;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < static_cast<unsigned>(W)) red_add_sys(P.flags[threadIdx.x] + 1, 1u);
    __syncthreads();
    if (threadIdx.x == 0) *done = 0;
}

// one thread waits until *flag >= target (bounded; error word on timeout)
__global__ void ep_wait_kernel(const uint32_t *flag, uint32_t target, uint64_t timeout_ns, int *err) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = clock64(), lim = timeout_cycles(timeout_ns);
    while (static_cast<int32_t>(ld_acquire_sys(flag) - target) < 0) {
        if (static_cast<uint64_t>(clock64()) - t0 > lim) {
            set_error(err, DERR_TIMEOUT_FULL);
            return;
        }
        __nanosleep(256);
    }
    __threadfence_system();
}

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool load_peers(const void *const *ptrs, int W, EpPeers &P) {
    if (W < 1 || W > EP_MAX_WORLD) return false;
    memset(&P, 0, sizeof(P));
    for (int r = 0; r < W; ++r) {
        P.x[r] = static_cast<float *>(const_cast<void *>(ptrs[0 * W + r]));
        P.ids[r] = static_cast<int32_t *>(const_cast<void *>(ptrs[1 * W + r]));
        P.src[r] = static_cast<int32_t *>(const_cast<void *>(ptrs[2 * W + r]));
        P.y_ret[r] = static_cast<float *>(const_cast<void *>(ptrs[3 * W + r]));
        P.flags[r] = static_cast<uint32_t *>(const_cast<void *>(ptrs[4 * W + r]));
        if (!P.x[r] || !P.ids[r] || !P.src[r] || !P.y_ret[r] || !P.flags[r]) return false;
        // rows move as float4: every peer row buffer must be 16-byte aligned
        if (!aligned16(P.x[r]) || !aligned16(P.y_ret[r])) return false;
    }
    return true;
}

int grid_for(int64_t warps) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (warps + 7) / 8;
    return static_cast<int>(blocks < 4 * n_sm ? (blocks > 0 ? blocks : 1) : 4 * n_sm);
}

}  // namespace

cudaError_t launch_ep_dispatch(const void *const *peer_ptrs, int W, int me, int cap, const int32_t *ids,
                               int n_entries, int k, int E, const float *x, int H, uint32_t *scratch, int *err,
                               cudaStream_t st) {
    EpPeers P;
    if (!load_peers(peer_ptrs, W, P) || H % 4 || !aligned16(x)) return cudaErrorInvalidValue;
    ep_dispatch_kernel<<<grid_for(n_entries), 256, 0, st>>>(P, W, me, cap, ids, n_entries, k, E, x, H, scratch,
                                                            scratch + EP_MAX_WORLD, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_return(const void *const *peer_ptrs, int W, int cap, const int32_t *ids, const int32_t *src,
                             const float *y, int H, uint32_t *scratch, cudaStream_t st) {
    EpPeers P;
    if (!load_peers(peer_ptrs, W, P) || H % 4 || !aligned16(y)) return cudaErrorInvalidValue;
    ep_return_kernel<<<grid_for(static_cast<int64_t>(W) * cap), 256, 0, st>>>(P, W, cap, ids, src, y, H,
                                                                              scratch + EP_MAX_WORLD + 1);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait(const uint32_t *flag, uint32_t target, uint64_t timeout_ns, int *err, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(flag, target, timeout_ns, err);
    return cudaGetLastError();
}

}  // namespace moe
