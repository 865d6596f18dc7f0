// moe_promote.cu -- promotion pass of the hot-expert cache on the GPU (see
// moe_promote.cuh for the policy and why it runs on the device).
//
// promote_kernel, one CTA of 1024 threads:
//   1. takes the step's counters (and clears them), advances the clock;
//   2. sorts the step's miss log in shared memory (bitonic) and reduces it to
//      distinct (tensor, expert) keys with their multiplicities;
//   3. decides every key's fate in parallel. A key whose admission state
//      plus multiplicity reaches two makes a promotion attempt; the attempt
//      succeeds when the expert is not resident and its tensor has a pool.
//      The n-th successful key in key order gets promotion index n; keys
//      past the 48th promotion are left untouched, as the reference stops
//      reading its log there; every other key's admission state becomes
//      (state + multiplicity) mod 2, and 0 for the key that made the 48th;
//   4. one warp per tensor with promotions picks the slots in key order: the
//      lowest free slot, else the slot whose expert has the oldest stamp
//      (ties to the lowest slot). It evicts (table entry back to the tagged
//      host address), installs the new expert and writes a copy job.
// promote_copy_kernel then copies the jobs' experts from pinned host memory
// into their slots. Both run on the caller's stream before the next decode.
#include "moe_promote.cuh"

namespace moe {

namespace {

constexpr uint32_t kPad = 0xFFFFFFFFu;

// In-place exclusive scan of v[0..n) (n <= 16 * 1024) by a 1024-thread block;
// returns the total. Thread t owns elements [16 t, 16 t + 16).
__device__ uint32_t block_exclusive_scan(uint32_t *v, int n, uint32_t *warp_sums) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int PER = 16;
    uint32_t local[PER], sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        local[i] = idx < n ? v[idx] : 0u;
        sum += local[i];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = warp_sums[lane];
        uint32_t wi = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t o = __shfl_up_sync(0xffffffffu, wi, off);
            if (lane >= off) wi += o;
        }
        warp_sums[lane] = wi - w;          // exclusive prefix of the warps
        if (lane == 31) warp_sums[32] = wi;
    }
    __syncthreads();
    uint32_t run = warp_sums[warp] + incl - sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        if (idx < n) v[idx] = run;
        run += local[i];
    }
    const uint32_t total = warp_sums[32];
    __syncthreads();
    return total;
}

// Ascending bitonic sort of v[0..P), P a power of two.
__device__ void block_bitonic_sort(uint32_t *v, int P) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int o = i ^ j;
                if (o > i) {
                    const uint32_t a = v[i], b = v[o];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) { v[i] = b; v[o] = a; }
                }
            }
            __syncthreads();
        }
    }
}

__global__ void __launch_bounds__(PROMOTE_THREADS, 1) promote_kernel(CacheDev *S, uint32_t *stats, uint32_t log_cap) {
    extern __shared__ __align__(16) uint32_t sm[];
    __shared__ uint32_t s_n, s_cut, s_evict;
    __shared__ uint32_t warp_sums[33];
    __shared__ int32_t s_list[PROMOTE_MAX];      // promotion index -> key index
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t cap_pow2 = 1u << (32 - __clz(static_cast<int>(log_cap > 1 ? log_cap - 1 : 1)));
    uint32_t *keys = sm;                         // [cap_pow2]: sorted log, then distinct keys
    uint32_t *start = sm + cap_pow2;             // [cap_pow2 + 1]: run starts
    uint32_t *succ = start + cap_pow2 + 1;       // [cap_pow2]: successful attempt flags -> prefix

    // ---- 1. counters of the finished step; the next launches stamp clock + 1
    if (tid == 0) {
        const uint32_t raw = stats[0], hits = stats[1];
        const uint32_t n = raw < log_cap ? raw : log_cap;
        s_n = n;
        S->steps += 1;
        S->hits += hits;
        S->misses += raw;
        S->overflow += raw - n;
        S->clock += 1;
        S->n_jobs = 0;
        s_evict = 0;
    }
    __syncthreads();
    const int n = static_cast<int>(s_n);
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += PROMOTE_THREADS) keys[i] = i < n ? stats[2 + i] : kPad;
    __syncthreads();
    if (tid == 0) { stats[0] = 0; stats[1] = 0; }
    if (n == 0) return;

    // ---- 2. sort; distinct keys and their run starts ------------------------
    block_bitonic_sort(keys, P);
    for (int i = tid; i < n; i += PROMOTE_THREADS) start[i] = (i == 0 || keys[i] != keys[i - 1]) ? 1u : 0u;
    __syncthreads();
    // flags -> positions; each thread keeps its elements' (key, flag) first
    constexpr int PER = 16;
    uint32_t mykey[PER], myflag[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        mykey[i] = idx < n ? keys[idx] : kPad;
        myflag[i] = idx < n ? start[idx] : 0u;
    }
    __syncthreads();
    const uint32_t nk = block_exclusive_scan(start, n, warp_sums);   // start[i] = position of run i
    uint32_t mypos[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) mypos[i] = (tid * PER + i) < n ? start[tid * PER + i] : 0u;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        if (idx < n && myflag[i]) {
            keys[mypos[i]] = mykey[i];
            start[mypos[i]] = static_cast<uint32_t>(idx);
        }
    }
    if (tid == 0) start[nk] = static_cast<uint32_t>(n);
    __syncthreads();

    // ---- 3. each key's attempt; promotion indices by scan --------------------
    const int n_tensors = S->n_tensors;
    const CacheTensorDev *reg = S->reg;
    for (uint32_t j = tid; j < nk; j += PROMOTE_THREADS) {
        const uint32_t key = keys[j], m = start[j + 1] - start[j];
        const int cid = static_cast<int>(key >> 12), e = static_cast<int>(key & 0xFFFu);
        uint32_t ok = 0;
        if (cid < n_tensors) {
            const CacheTensorDev &T = reg[cid];
            if (T.live && e < T.n_experts && T.seen[e] + m >= 2u && T.n_slots > 0 && T.slot_of[e] < 0) ok = 1;
        }
        succ[j] = ok;
    }
    __syncthreads();
    // keep the flags: the scan overwrites them (thread t owns keys 16 t ..)
    uint32_t myok[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) myok[i] = (tid * PER + i) < static_cast<int>(nk) ? succ[tid * PER + i] : 0u;
    __syncthreads();
    const uint32_t total = block_exclusive_scan(succ, static_cast<int>(nk), warp_sums);
    if (tid == 0) s_cut = kPad;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const uint32_t j = static_cast<uint32_t>(tid * PER + i);
        if (j < nk && myok[i] && succ[j] < static_cast<uint32_t>(PROMOTE_MAX)) {
            s_list[succ[j]] = static_cast<int32_t>(j);
            if (succ[j] == static_cast<uint32_t>(PROMOTE_MAX - 1)) s_cut = j;   // the 48th promotion
        }
    }
    __syncthreads();
    const uint32_t cut = s_cut;
    const int n_prom = static_cast<int>(total < static_cast<uint32_t>(PROMOTE_MAX) ? total : PROMOTE_MAX);
    // admission states: keys up to the cut; the key of the 48th promotion ends at 0
    for (uint32_t j = tid; j < nk; j += PROMOTE_THREADS) {
        if (cut != kPad && j > cut) continue;
        const uint32_t key = keys[j], m = start[j + 1] - start[j];
        const int cid = static_cast<int>(key >> 12), e = static_cast<int>(key & 0xFFFu);
        if (cid >= n_tensors) continue;
        const CacheTensorDev &T = reg[cid];
        if (!T.live || e >= T.n_experts) continue;
        const uint8_t now = j == cut ? 0 : static_cast<uint8_t>((T.seen[e] + m) & 1u);
        if (T.seen[e] != now) T.seen[e] = now;
    }

    // ---- 4. slots: one warp per run of promotions of one tensor --------------
    for (int g = warp; g < n_prom; g += PROMOTE_THREADS / 32) {
        const int cid = static_cast<int>(keys[s_list[g]] >> 12);
        if (g > 0 && static_cast<int>(keys[s_list[g - 1]] >> 12) == cid) continue;   // not the head of its run
        const CacheTensorDev &T = reg[cid];
        for (int p = g; p < n_prom && static_cast<int>(keys[s_list[p]] >> 12) == cid; ++p) {
            const int e = static_cast<int>(keys[s_list[p]] & 0xFFFu);
            // lowest free slot
            int slot = -1;
            for (int base = 0; base < T.n_slots && slot < 0; base += 32) {
                const int s = base + lane;
                const unsigned fr = __ballot_sync(0xffffffffu, s < T.n_slots && T.expert_of[s] < 0);
                if (fr) slot = base + __ffs(fr) - 1;
            }
            int victim = -1;
            if (slot < 0) {
                // oldest stamp, ties to the lowest slot
                uint32_t best = kPad;
                int bs = -1;
                for (int s = lane; s < T.n_slots; s += 32) {
                    const int v = T.expert_of[s];
                    const uint32_t stamp = v >= 0 ? T.stamps[v] : 0u;
                    if (stamp < best) { best = stamp; bs = s; }
                }
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) {
                    const uint32_t ob = __shfl_xor_sync(0xffffffffu, best, off);
                    const int os = __shfl_xor_sync(0xffffffffu, bs, off);
                    if (ob < best || (ob == best && os >= 0 && (bs < 0 || os < bs))) { best = ob; bs = os; }
                }
                slot = bs;   // -1 only if every stamp were 0xFFFFFFFF (2^32 steps of the clock)
                if (slot >= 0) victim = T.expert_of[slot];
            }
            if (lane == 0 && slot >= 0) {
                if (victim >= 0) {
                    T.slot_of[victim] = -1;
                    T.tbl[victim] = reinterpret_cast<char *>(
                        reinterpret_cast<uintptr_t>(T.host + static_cast<uint64_t>(victim) * T.expert_bytes) | 1u);
                    atomicAdd(&s_evict, 1u);
                }
                char *dst = T.pool + static_cast<uint64_t>(slot) * T.expert_bytes;
                T.expert_of[slot] = e;
                T.slot_of[e] = slot;
                T.tbl[e] = dst;
                S->jobs[p] = PromoteJob{T.host + static_cast<uint64_t>(e) * T.expert_bytes, dst, T.expert_bytes};
            }
            __syncwarp();
        }
    }
    __syncthreads();
    if (tid == 0) {
        S->n_jobs = static_cast<uint32_t>(n_prom);
        S->promotions += static_cast<unsigned long long>(n_prom);
        S->evictions += s_evict;
    }
}

// Copies this step's promoted experts from pinned host memory (read over the
// host link) into their pool slots: 16-byte words when both ends and the size
// allow, else bytes. Every CTA takes every job's chunks with its index.
__global__ void __launch_bounds__(256) promote_copy_kernel(const CacheDev *S) {
    const uint32_t n_jobs = *reinterpret_cast<const volatile uint32_t *>(&S->n_jobs);
    constexpr uint64_t CHUNK = 32768;
    for (uint32_t j = 0; j < n_jobs; ++j) {
        const PromoteJob job = S->jobs[j];
        const uint64_t n_chunks = (job.bytes + CHUNK - 1) / CHUNK;
        const bool v16 = ((reinterpret_cast<uintptr_t>(job.src) | reinterpret_cast<uintptr_t>(job.dst) | job.bytes) & 15u) == 0;
        for (uint64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
            const uint64_t lo = c * CHUNK, hi = lo + CHUNK < job.bytes ? lo + CHUNK : job.bytes;
            if (v16) {
                const uint4 *s = reinterpret_cast<const uint4 *>(job.src + lo);
                uint4 *d = reinterpret_cast<uint4 *>(job.dst + lo);
                for (uint64_t i = threadIdx.x; i < (hi - lo) / 16; i += blockDim.x) d[i] = s[i];
            } else {
                for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) job.dst[i] = job.src[i];
            }
        }
    }
}

}  // namespace

size_t promote_smem_bytes(uint32_t log_cap) {
    uint32_t p = 1;
    while (p < log_cap) p <<= 1;
    return sizeof(uint32_t) * (3ull * p + 1);
}

cudaError_t launch_promote(CacheDev *state, uint32_t *stats, uint32_t log_cap, cudaStream_t st) {
    if (log_cap > 16u * PROMOTE_THREADS) return cudaErrorInvalidValue;
    const size_t smem = promote_smem_bytes(log_cap);
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(promote_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    promote_kernel<<<1, PROMOTE_THREADS, smem, st>>>(state, stats, log_cap);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    promote_copy_kernel<<<2 * n_sm, 256, 0, st>>>(state);
    return cudaGetLastError();
}

}  // namespace moe
