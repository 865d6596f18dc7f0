// moe_promote.cuh -- the hot-expert cache's promotion pass, run on the GPU.
//
// The cache policy is the reference's (kernels/moe-cache.cu:628-775 of
// Zapdev-labs/a6000-custom-kernels): a missed expert is admitted on its
// second sighting, at most 48 experts are promoted per step, a full pool
// evicts the resident expert with the oldest stamp (ties to the lowest slot),
// and one step's misses are taken in (tensor << 12 | expert) order. The
// reference runs it on the host after a blocking copy of the miss log and a
// stream synchronisation, and syncs again for the stamps on the first
// eviction of a tensor. Here the whole pass is two kernels on the caller's
// stream: promote_kernel decides every promotion and patches the pointer
// tables, slot maps and admission bits in device memory, and
// promote_copy_kernel moves the promoted experts from pinned host memory
// into their pool slots. The host never waits, and a step can be captured
// in a CUDA graph together with the decode launches around it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

constexpr int PROMOTE_MAX = 48;        // promotions per step (reference :37)
constexpr int PROMOTE_THREADS = 1024;

// One registered expert tensor as the promotion pass sees it; the registry is
// an array of these indexed by tensor id (the id packed in the miss log).
struct CacheTensorDev {
    char **tbl;              // [n_experts] tagged pointers read by the kernels (bit 0: host memory)
    const uint32_t *stamps;  // [n_experts] clock of the last launch that used the expert
    int32_t *slot_of;        // [n_experts] pool slot holding the expert, or -1
    int32_t *expert_of;      // [n_slots] expert held by the slot, or -1
    uint8_t *seen;           // [n_experts] admission state: 1 = missed once since its last admission
    const char *host;        // the caller's (pinned host) copy of expert 0
    char *pool;              // slot 0 of the HBM pool
    uint64_t expert_bytes;
    int32_t n_experts, n_slots;
    int32_t live;            // 0: retired, or HBM-resident (no pool): its log entries are skipped
    int32_t pad_;
};

struct PromoteJob {
    const char *src;         // pinned host memory
    char *dst;               // pool slot
    uint64_t bytes;
};

// Device-resident state of the cache: the registry, the launch clock the
// kernels stamp with, running totals and this step's copy list. Fixed
// address for the life of the cache, so captured graphs stay valid.
struct CacheDev {
    CacheTensorDev *reg;
    int32_t n_tensors;
    uint32_t clock;
    unsigned long long steps, hits, misses, promotions, evictions, overflow;
    uint32_t n_jobs;
    uint32_t pad_;
    PromoteJob jobs[PROMOTE_MAX];
};

// stats: [0] misses of the step, [1] hits, [2..2+log_cap) the miss log.
size_t promote_smem_bytes(uint32_t log_cap);
cudaError_t launch_promote(CacheDev *state, uint32_t *stats, uint32_t log_cap, cudaStream_t st);

}  // namespace moe
