// moe_cache.cu -- host side of the hot-expert cache and the C ABI.
//
// Serves the reference's boundary (kernels/moe-cache.cuh:15-40 of
// Zapdev-labs/a6000-custom-kernels) with a B200 design of its own:
//   * Each registered expert tensor owns one device block holding its
//     pointer table, stamps, slot maps and admission bits, plus an HBM pool
//     when its experts live in pinned host memory. Tensors already in HBM
//     (the normal case on a 180 GB B200) get a table of direct pointers and
//     no pool; the promotion pass skips them.
//   * The promotion step runs on the GPU (moe_promote.cu): the host enqueues
//     two kernels and never waits, where the reference copies the miss log
//     back and synchronises the stream every step (moe-cache.cu:677-678)
//     and again for the stamps on an eviction (:641-642). The policy is the
//     reference's: second-sighting admission, at most 48 promotions per
//     step, LRU eviction with ties to the lowest slot, misses taken in
//     (tensor << 12 | expert) order (the reference takes them in atomicAdd
//     arrival order, which depends on block scheduling; sorted order is one
//     of the orders it can produce and makes the state reproducible).
//   * Pool sizing follows the reference's rule (:542-561): the configured
//     slot count, capped by the budget left, by free HBM minus 2 GiB and by
//     the expert count; seeding fills slots 0.. in seed-file order (:584-609).
//   * Every entry point returns a status instead of aborting; a gate tensor
//     without a table is read at its expert's offset (the reference reads
//     expert 0 there, :200).
#include <algorithm>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "moe_aux.h"
#include "moe_cache_b200.h"
#include "moe_gemv.cuh"
#include "moe_layer2.cuh"
#include "moe_stack.cuh"
#include "moe_mmq.cuh"
#include "moe_promote.cuh"

namespace {

constexpr uint32_t kLogCap = 16382;            // miss-log entries per step (the reference keeps 8190)
constexpr int kLogWords = 2 + static_cast<int>(kLogCap);
constexpr size_t kHbmReserve = 2ull << 30;     // free HBM a pool never takes
constexpr int kMaxExperts = 4096;              // 12 bits of the miss-log packing

// One expert tensor known to the cache (keyed by its data pointer).
struct Tensor {
    int32_t id = -1;               // registry index, packed into miss-log entries
    int type = 0;
    const char *data = nullptr;
    uint64_t expert_bytes = 0, row_bytes = 0;
    int64_t rows = 0, cols = 0;
    int n_experts = 0, n_slots = 0;
    bool tiered = false;           // experts in pinned host memory, served through a pool
    bool retired = false;          // its address now holds another tensor
    std::string name;
    // device block: table, stamps, slot map, slot owners, admission bits
    char *block = nullptr;
    char **table = nullptr;
    uint32_t *stamps = nullptr;
    int32_t *slot_map = nullptr, *slot_owner = nullptr;
    uint8_t *seen = nullptr;
    char *pool = nullptr;
};

struct Cache {
    // configuration (environment or moe_b200_configure)
    bool enabled = false, env_read = false, configured = false;
    int slots = 320;
    size_t budget = 30ull << 30;
    bool claim_device = true;
    bool debug = false;
    int layer_fused = 1;          // 0: four launches; 1: per-expert-group kernel; 2: grid-exchange kernel
    std::string seed_path;
    // registry
    std::unordered_map<const char *, Tensor *> by_ptr;
    std::vector<Tensor *> tensors;
    size_t pool_bytes = 0;
    bool any_tiered = false;
    // seed lists by tensor name, read on first registration
    std::unordered_map<std::string, std::vector<int>> seeds;
    bool seeds_read = false;
    // device side
    int device = -1;
    moe::CacheDev *dev = nullptr;           // registry pointer, clock, totals, copy jobs
    moe::CacheTensorDev *d_reg = nullptr;   // registry array
    int reg_cap = 0;
    uint32_t *d_log = nullptr;              // [0] misses, [1] hits, [2..] miss log
    int *d_err = nullptr;
    uint64_t timeout_ns_ep = 2000000000ull;       // expert-parallel arrival waits
    uint64_t timeout_ns_kernel = 2000000000ull;   // waits inside the GEMV / layer / prefill kernels
    uint64_t idle_steps = 0;                // step calls with nothing tiered (no kernel launched)
    uint64_t step_calls = 0;
    std::unordered_map<const void *, int> ptr_kind;   // 1 host, 2 device, 0 other
};

Cache g;
std::recursive_mutex g_mu;
thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return fail(MOE_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

int type_size(int t) {
    switch (t) {
        case MOE_TYPE_Q4_0: return 18;
        case MOE_TYPE_Q5_0: return 22;
        case MOE_TYPE_Q8_0: return 34;
        case MOE_TYPE_Q2_K: return 84;
        case MOE_TYPE_Q3_K: return 110;
        case MOE_TYPE_Q4_K: return 144;
        case MOE_TYPE_Q5_K: return 176;
        case MOE_TYPE_Q6_K: return 210;
        default: return 0;
    }
}
int blck_size(int t) { return (t >= MOE_TYPE_Q2_K && t <= MOE_TYPE_Q6_K) ? 256 : 32; }

// the eight formats of the reference's op (moe-cache.cu:407-421)
bool type_supported(int t) { return type_size(t) != 0; }

int env_int(const char *n, int fb) { const char *s = getenv(n); return s ? atoi(s) : fb; }
double env_double(const char *n, double fb) { const char *s = getenv(n); return s ? atof(s) : fb; }

// The drop-in's configuration variables (names as in moe-cache.cu:345-363),
// read once unless moe_b200_configure set the configuration.
void read_env() {
    if (g.env_read) return;
    const char *on = getenv("GGML_CUDA_MOE_CACHE");
    g.enabled = on && on[0] && on[0] != '0';
    g.slots = std::max(0, env_int("GGML_CUDA_MOE_CACHE_SLOTS", g.slots));
    const double gib = env_double("GGML_CUDA_MOE_CACHE_BUDGET_GB", 0.0);
    if (gib > 0) g.budget = static_cast<size_t>(gib * 1073741824.0);
    const char *seed = getenv("GGML_CUDA_MOE_CACHE_SEED");
    g.seed_path = seed ? seed : "";
    g.claim_device = env_int("GGML_CUDA_MOE_CACHE_DEVICE", 1) != 0;
    g.debug = getenv("GGML_CUDA_MOE_CACHE_DEBUG") != nullptr;
    g.layer_fused = std::min(2, std::max(0, env_int("GGML_CUDA_MOE_LAYER_FUSED", 1)));
    g.env_read = true;
    if (g.enabled && g.debug)
        fprintf(stderr, "[moe_b200] cache on: %d slots per tensor, %.1f GiB pool budget\n", g.slots,
                static_cast<double>(g.budget) / 1073741824.0);
}

// 1 = pinned host, 2 = device memory of the current device, 0 = neither
int ptr_kind(const void *p) {
    auto it = g.ptr_kind.find(p);
    if (it != g.ptr_kind.end()) return it->second;
    cudaPointerAttributes attrs;
    int kind = 0;
    if (cudaPointerGetAttributes(&attrs, p) == cudaSuccess) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (attrs.type == cudaMemoryTypeHost) kind = 1;
        else if (attrs.type == cudaMemoryTypeDevice && attrs.device == dev) kind = 2;
    } else {
        cudaGetLastError();
    }
    g.ptr_kind[p] = kind;
    return kind;
}

bool contiguous(const moe_tensor *t) {
    const uint64_t ts = static_cast<uint64_t>(type_size(t->type));
    const int64_t bs = blck_size(t->type);
    if (t->ne[0] % bs) return false;
    return t->nb[0] == ts && t->nb[1] == ts * static_cast<uint64_t>(t->ne[0] / bs) &&
           t->nb[2] == t->nb[1] * static_cast<uint64_t>(t->ne[1]) && t->nb[3] == t->nb[2] * static_cast<uint64_t>(t->ne[2]);
}

// The reference's eligibility test (moe-cache.cu:442-469), widened to
// tensors in device memory (HBM-resident experts).
int wants_locked(const moe_tensor *src0) {
    read_env();
    if (!g.enabled || !src0 || !src0->data) return 0;
    if (src0->flags & (MOE_TENSOR_NO_BUFFER | MOE_TENSOR_VIEW)) return 0;
    const int kind = ptr_kind(src0->data);
    if (kind == 0 || (kind == 2 && !g.claim_device)) return 0;
    if (!type_supported(src0->type) || src0->ne[2] < 2 || src0->ne[3] != 1) return 0;
    return contiguous(src0) ? 1 : 0;
}

uint32_t *clock_ptr() {
    return reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(g.dev) + offsetof(moe::CacheDev, clock));
}

// The cache's device state on the current device, made on first use.
int ensure_device() {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (g.dev) {
        if (dev != g.device) return fail(MOE_ERR_STATE, "moe-cache state belongs to device %d, called on %d", g.device, dev);
        return MOE_OK;
    }
    CK(cudaMalloc(&g.dev, sizeof(moe::CacheDev)));
    CK(cudaMemset(g.dev, 0, sizeof(moe::CacheDev)));
    CK(cudaMalloc(&g.d_log, sizeof(uint32_t) * kLogWords));
    CK(cudaMemset(g.d_log, 0, sizeof(uint32_t) * kLogWords));
    CK(cudaMalloc(&g.d_err, sizeof(int)));
    CK(cudaMemset(g.d_err, 0, sizeof(int)));
    g.device = dev;
    return MOE_OK;
}

// ---- seed lists -------------------------------------------------------------
// One line per tensor: "<tensor name> <id>,<id>,..." (the format written by
// the reference's tools/make_seed.py). Ids are read up to the first token
// that is not an integer.
bool parse_id(const std::string &tok, int *out) {
    size_t a = 0, b = tok.size();
    while (a < b && isspace(static_cast<unsigned char>(tok[a]))) ++a;
    while (b > a && isspace(static_cast<unsigned char>(tok[b - 1]))) --b;
    if (a == b) return false;
    size_t i = a;
    if (tok[i] == '+' || tok[i] == '-') ++i;
    if (i == b) return false;
    long v = 0;
    for (; i < b; ++i) {
        if (tok[i] < '0' || tok[i] > '9') return false;
        v = v * 10 + (tok[i] - '0');
        if (v > (1L << 30)) return false;
    }
    *out = static_cast<int>(tok[a] == '-' ? -v : v);
    return true;
}

void read_seeds() {
    if (g.seeds_read) return;
    g.seeds_read = true;
    if (g.seed_path.empty()) return;
    std::ifstream in(g.seed_path);
    if (!in) {
        fprintf(stderr, "[moe_b200] no seed file at %s; pools start empty\n", g.seed_path.c_str());
        return;
    }
    std::string line;
    while (std::getline(in, line)) {
        if (!line.empty() && line.back() == '\r') line.pop_back();
        const size_t sp = line.find(' ');
        if (sp == std::string::npos) continue;
        std::vector<int> ids;
        for (size_t pos = sp + 1;;) {
            const size_t comma = line.find(',', pos);
            int id = 0;
            if (!parse_id(line.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos), &id)) break;
            ids.push_back(id);
            if (comma == std::string::npos) break;
            pos = comma + 1;
        }
        g.seeds[line.substr(0, sp)] = std::move(ids);
    }
    if (g.debug) fprintf(stderr, "[moe_b200] seed lists for %zu tensors from %s\n", g.seeds.size(), g.seed_path.c_str());
}

// ---- registry ---------------------------------------------------------------
char *tagged_host(const char *p) { return reinterpret_cast<char *>(reinterpret_cast<uintptr_t>(p) | 1u); }
size_t round_up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Pool slots for a tiered tensor: the configured count, capped by the budget
// left, by free HBM beyond the reserve, and by the expert count.
int pool_slots(const Tensor &t) {
    if (!t.tiered) return 0;
    int64_t s = g.slots;
    const size_t budget_left = g.budget > g.pool_bytes ? g.budget - g.pool_bytes : 0;
    s = std::min<int64_t>(s, static_cast<int64_t>(budget_left / t.expert_bytes));
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { cudaGetLastError(); return -1; }
    const size_t usable = free_b > kHbmReserve ? free_b - kHbmReserve : 0;
    s = std::min<int64_t>(s, static_cast<int64_t>(usable / t.expert_bytes));
    return static_cast<int>(std::min<int64_t>(s, t.n_experts));
}

// The registry array has room for tensor id `id` (grows by doubling; the
// promotion pass reads it, so the device is idle while it moves).
int reserve_registry(int id) {
    if (id < g.reg_cap) return MOE_OK;
    const int cap = std::max(256, 2 * g.reg_cap);
    moe::CacheTensorDev *fresh = nullptr;
    CK(cudaDeviceSynchronize());
    CK(cudaMalloc(&fresh, sizeof(moe::CacheTensorDev) * cap));
    CK(cudaMemset(fresh, 0, sizeof(moe::CacheTensorDev) * cap));
    if (g.d_reg) CK(cudaMemcpy(fresh, g.d_reg, sizeof(moe::CacheTensorDev) * g.reg_cap, cudaMemcpyDeviceToDevice));
    CK(cudaMemcpy(reinterpret_cast<char *>(g.dev) + offsetof(moe::CacheDev, reg), &fresh, sizeof(fresh),
                  cudaMemcpyHostToDevice));
    if (g.d_reg) CK(cudaFree(g.d_reg));
    g.d_reg = fresh;
    g.reg_cap = cap;
    return MOE_OK;
}

int publish(const Tensor &t, cudaStream_t st) {
    moe::CacheTensorDev d{};
    d.tbl = t.table;
    d.stamps = t.stamps;
    d.slot_of = t.slot_map;
    d.expert_of = t.slot_owner;
    d.seen = t.seen;
    d.host = t.data;
    d.pool = t.pool;
    d.expert_bytes = t.expert_bytes;
    d.n_experts = t.n_experts;
    d.n_slots = t.n_slots;
    d.live = (t.tiered && !t.retired) ? 1 : 0;
    CK(cudaMemcpyAsync(g.d_reg + t.id, &d, sizeof(d), cudaMemcpyHostToDevice, st));
    const int32_t n = static_cast<int32_t>(g.tensors.size());
    CK(cudaMemcpyAsync(reinterpret_cast<char *>(g.dev) + offsetof(moe::CacheDev, n_tensors), &n, sizeof(n),
                       cudaMemcpyHostToDevice, st));
    return MOE_OK;
}

void release(Tensor *t) {
    cudaFree(t->block);
    cudaFree(t->pool);
    t->block = t->pool = nullptr;
    t->table = nullptr;
    t->stamps = nullptr;
    t->slot_map = t->slot_owner = nullptr;
    t->seen = nullptr;
}

// A different tensor now lives at this tensor's address: free its device
// state (after the device is idle) and mark it dead. It keeps its id so
// the ids of later tensors, packed into miss-log entries, stay valid.
int retire(Tensor *t) {
    CK(cudaDeviceSynchronize());
    release(t);
    g.pool_bytes -= static_cast<size_t>(t->n_slots) * t->expert_bytes;
    t->n_slots = 0;
    t->retired = true;
    g.by_ptr.erase(t->data);
    moe::CacheTensorDev dead{};
    CK(cudaMemcpy(g.d_reg + t->id, &dead, sizeof(dead), cudaMemcpyHostToDevice));
    return MOE_OK;
}

// The cache's record of src0, registering it on first sight: device block,
// pool, initial table (tagged host addresses or direct device addresses),
// seeded slots, and its registry entry for the promotion pass.
int enroll(const moe_tensor *src0, cudaStream_t st, Tensor **out) {
    int rc = ensure_device();
    if (rc) return rc;
    const char *key = static_cast<const char *>(src0->data);
    auto hit = g.by_ptr.find(key);
    if (hit != g.by_ptr.end()) {
        Tensor *t = hit->second;
        if (t->type == src0->type && t->n_experts == src0->ne[2] && t->expert_bytes == src0->nb[2] &&
            t->row_bytes == src0->nb[1] && t->rows == src0->ne[1] && t->cols == src0->ne[0]) {
            *out = t;
            return MOE_OK;
        }
        rc = retire(t);
        if (rc) return rc;
    }
    if (src0->ne[2] > kMaxExperts) return fail(MOE_ERR_UNSUPPORTED, "more than %d experts", kMaxExperts);

    Tensor *t = new Tensor();
    t->id = static_cast<int32_t>(g.tensors.size());
    t->type = src0->type;
    t->data = key;
    t->expert_bytes = src0->nb[2];
    t->row_bytes = src0->nb[1];
    t->rows = src0->ne[1];
    t->cols = src0->ne[0];
    t->n_experts = static_cast<int>(src0->ne[2]);
    t->tiered = ptr_kind(src0->data) == 1;
    t->name = src0->name ? src0->name : "";
    t->n_slots = pool_slots(*t);
    if (t->n_slots < 0) { delete t; return fail(MOE_ERR_CUDA, "cudaMemGetInfo failed"); }
    rc = reserve_registry(t->id);
    if (rc) { delete t; return rc; }

    const size_t E = static_cast<size_t>(t->n_experts);
    const size_t o_stamps = round_up256(sizeof(char *) * E), o_map = o_stamps + round_up256(4 * E),
                 o_owner = o_map + round_up256(4 * E), o_seen = o_owner + round_up256(4 * (t->n_slots + 1)),
                 bytes = o_seen + round_up256(E);
    if (cudaMalloc(&t->block, bytes) != cudaSuccess ||
        (t->n_slots > 0 && cudaMalloc(&t->pool, static_cast<size_t>(t->n_slots) * t->expert_bytes) != cudaSuccess)) {
        cudaGetLastError();
        release(t);
        delete t;
        return fail(MOE_ERR_OOM, "cache allocation for %s failed", src0->name ? src0->name : "<tensor>");
    }
    t->table = reinterpret_cast<char **>(t->block);
    t->stamps = reinterpret_cast<uint32_t *>(t->block + o_stamps);
    t->slot_map = reinterpret_cast<int32_t *>(t->block + o_map);
    t->slot_owner = reinterpret_cast<int32_t *>(t->block + o_owner);
    t->seen = reinterpret_cast<uint8_t *>(t->block + o_seen);
    g.pool_bytes += static_cast<size_t>(t->n_slots) * t->expert_bytes;
    g.any_tiered |= t->tiered;

    // initial state on the host, then one upload per array
    std::vector<char *> table(E);
    std::vector<int32_t> slot_map(E, -1), slot_owner(static_cast<size_t>(t->n_slots), -1);
    for (size_t x = 0; x < E; ++x) {
        const char *p = t->data + x * t->expert_bytes;
        table[x] = t->tiered ? tagged_host(p) : const_cast<char *>(p);
    }
    read_seeds();
    const auto seed = g.seeds.find(t->name);
    int filled = 0;
    if (seed != g.seeds.end()) {
        for (const int x : seed->second) {
            if (filled == t->n_slots) break;
            if (x < 0 || x >= t->n_experts || slot_map[x] >= 0) continue;
            char *slot = t->pool + static_cast<size_t>(filled) * t->expert_bytes;
            CK(cudaMemcpyAsync(slot, t->data + static_cast<size_t>(x) * t->expert_bytes, t->expert_bytes,
                               cudaMemcpyHostToDevice, st));
            table[x] = slot;
            slot_map[x] = filled;
            slot_owner[filled] = x;
            ++filled;
        }
    }
    CK(cudaMemsetAsync(t->stamps, 0, 4 * E, st));
    CK(cudaMemsetAsync(t->seen, 0, E, st));
    CK(cudaMemcpyAsync(t->slot_map, slot_map.data(), 4 * E, cudaMemcpyHostToDevice, st));
    if (t->n_slots > 0)
        CK(cudaMemcpyAsync(t->slot_owner, slot_owner.data(), 4 * static_cast<size_t>(t->n_slots), cudaMemcpyHostToDevice, st));
    // the table goes last: no kernel reads a slot before its expert is copied
    CK(cudaMemcpyAsync(t->table, table.data(), sizeof(char *) * E, cudaMemcpyHostToDevice, st));
    g.by_ptr[key] = t;
    g.tensors.push_back(t);
    rc = publish(*t, st);
    if (rc) return rc;
    // the host vectors above are pageable: the copies have taken them by now
    if (g.debug)
        fprintf(stderr, "[moe_b200] tensor %d %s: type %d, %d experts of %llu B, %s, %d slots (%d seeded)\n", t->id,
                t->name.c_str(), t->type, t->n_experts, static_cast<unsigned long long>(t->expert_bytes),
                t->tiered ? "pinned host memory" : "HBM", t->n_slots, filled);
    *out = t;
    return MOE_OK;
}

// ---- the step between graphs ---------------------------------------------------
int step_locked(cudaStream_t st) {
    if (!g.enabled || g.tensors.empty()) return MOE_OK;
    if (!g.any_tiered) { g.idle_steps++; return MOE_OK; }
    CK(moe::launch_promote(g.dev, g.d_log, kLogCap, st));
    if (g.debug && ++g.step_calls % 64 == 0) {
        moe::CacheDev s;
        CK(cudaStreamSynchronize(st));
        CK(cudaMemcpy(&s, g.dev, sizeof(s), cudaMemcpyDeviceToHost));
        fprintf(stderr, "[moe_b200] after %llu steps: %llu hits, %llu misses, %llu promoted, %llu evicted\n",
                s.steps, s.hits, s.misses, s.promotions, s.evictions);
    }
    return MOE_OK;
}

void free_all() {
    if (g.dev) cudaDeviceSynchronize();
    for (Tensor *t : g.tensors) {
        release(t);
        delete t;
    }
    g.tensors.clear();
    g.by_ptr.clear();
    cudaFree(g.dev);
    cudaFree(g.d_reg);
    cudaFree(g.d_log);
    cudaFree(g.d_err);
    g.dev = nullptr;
    g.d_reg = nullptr;
    g.reg_cap = 0;
    g.d_log = nullptr;
    g.d_err = nullptr;
    g.device = -1;
    g.pool_bytes = 0;
    g.any_tiered = false;
    g.seeds.clear();
    g.seeds_read = false;
    g.ptr_kind.clear();
    g.idle_steps = g.step_calls = 0;
}

// common GEMV argument setup for the boundary call and the layer path
struct MmvqCall {
    const moe_tensor *src0 = nullptr;
    const moe_tensor *gate = nullptr;            // fusion host gate tensor
    const moe_fusion_device *fd = nullptr;
    const void *src1 = nullptr;
    int src1_type = MOE_TYPE_Q8_1;
    const int32_t *ids = nullptr;
    float *dst = nullptr;
    int64_t ne00 = 0, ne01 = 0, ncols_dst = 0, s01 = 0;
    int64_t nchannels_y = 1, nchannels_dst = 0, stride_col_y = 0, stride_col_dst = 0;
    int64_t stride_channel_y = 0, stride_channel_dst = 0, ids_stride = 0;
    const void *shared_y = nullptr;               // layer path: shared-block activations
    int64_t shared_y_stride_col = 0;
    int64_t id_offset = 0;                        // expert-parallel: first expert of this GPU
    int skip_foreign = 0;                         // expert-parallel: other GPUs' ids are skipped
    int host_only = 0;                            // only picks of host-resident experts (prefill split)
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int run_mmvq(const MmvqCall &c, cudaStream_t stream) {
    const moe_tensor *src0 = c.src0;
    if (!src0 || !src0->data || !c.src1 || !c.ids || !c.dst) return fail(MOE_ERR_INVALID, "null argument");
    if (!type_supported(src0->type)) return fail(MOE_ERR_UNSUPPORTED, "moe-cache: unsupported expert type %d", src0->type);
    if (!contiguous(src0)) return fail(MOE_ERR_UNSUPPORTED, "expert tensor is not contiguous");
    if (c.src1_type != MOE_TYPE_Q8_1 && c.src1_type != MOE_TYPE_F32) return fail(MOE_ERR_UNSUPPORTED, "src1 must be Q8_1 or F32");
    if (c.ne00 != src0->ne[0] || c.ne01 != src0->ne[1]) return fail(MOE_ERR_INVALID, "ne00/ne01 do not match src0");
    if (c.nchannels_y < 1) return fail(MOE_ERR_INVALID, "nchannels_y < 1");
    // 16-byte aligned bases (ggml aligns tensor data to 32 bytes) keep every
    // shared-memory word load of the GEMV aligned
    if (!aligned16(src0->data)) return fail(MOE_ERR_UNSUPPORTED, "expert tensor data must be 16-byte aligned");
    if (c.fd && ((c.fd->gate && !aligned16(c.fd->gate)) || (c.fd->shared_up && !aligned16(c.fd->shared_up)) ||
                 (c.fd->shared_gate && !aligned16(c.fd->shared_gate))))
        return fail(MOE_ERR_UNSUPPORTED, "gate / shared expert data must be 16-byte aligned");
    Tensor *e = nullptr;
    int rc = enroll(src0, stream, &e);
    if (rc) return rc;
    const moe_fusion_device *fd = c.fd;
    const bool use_gate = fd && fd->gate;
    Tensor *ge = nullptr;
    if (use_gate && c.gate && wants_locked(c.gate)) {
        if (c.gate->type != src0->type || c.gate->ne[0] != src0->ne[0] || c.gate->ne[1] != src0->ne[1])
            return fail(MOE_ERR_UNSUPPORTED, "fused gate must match the up tensor's type and shape");
        rc = enroll(c.gate, stream, &ge);
        if (rc) return rc;
    }
    moe::GemvArgs a{};
    a.tbl = e->table;
    a.stamps = e->stamps;
    a.cache_id = e->id;
    a.use_gate = use_gate ? 1 : 0;
    a.has_fusion = fd && (fd->gate || fd->x_bias || fd->gate_bias || fd->x_scale || fd->gate_scale) ? 1 : 0;
    const bool tma_main = (src0->nb[2] % 16) == 0;
    a.tma_main = tma_main;
    if (use_gate) {
        if (ge) {
            a.tbl_gate = ge->table;
            a.stamps_gate = ge->stamps;
            a.cache_id_gate = ge->id;
            a.tma_gate = aligned16(ge->data) && (ge->expert_bytes % 16) == 0;
        } else {
            a.gate_dense = static_cast<const char *>(fd->gate);
            a.gate_expert_bytes = src0->nb[2];
            a.tma_gate = aligned16(fd->gate) && (src0->nb[2] % 16) == 0 && ptr_kind(fd->gate) == 2;
        }
        a.x_bias = fd->x_bias;
        a.gate_bias = fd->gate_bias;
    } else if (fd) {
        a.x_bias = fd->x_bias;
    }
    if (fd) {
        a.glu_op = fd->glu_op;
        a.glu_limit = fd->glu_limit;
        if (fd->shared_up) {
            if (use_gate && !fd->shared_gate) return fail(MOE_ERR_INVALID, "shared expert needs shared_gate with a fused gate");
            a.shared_up = static_cast<const char *>(fd->shared_up);
            a.shared_gate = use_gate ? static_cast<const char *>(fd->shared_gate) : nullptr;
            a.shared_dst = fd->shared_dst;
            a.shared_stride_col_dst = fd->shared_stride_col_dst;
            const uint64_t mat = src0->nb[2];
            a.tma_shared = aligned16(fd->shared_up) && (!use_gate || aligned16(fd->shared_gate)) && (mat % 16) == 0 &&
                           ptr_kind(fd->shared_up) == 2 && (!use_gate || ptr_kind(fd->shared_gate) == 2);
        }
    }
    a.shared_y = c.shared_y;
    a.shared_y_stride_col = c.shared_y_stride_col;
    a.stats = g.d_log;
    a.clock = clock_ptr();
    a.log_cap = kLogCap;
    a.y = c.src1;
    a.stride_col_y = c.stride_col_y;
    a.stride_channel_y = c.stride_channel_y;
    a.nchannels_y = static_cast<int32_t>(c.nchannels_y);
    a.ids = c.ids;
    a.ids_stride = c.ids_stride;
    a.id_offset = static_cast<int32_t>(c.id_offset);
    a.skip_foreign = c.skip_foreign;
    a.host_only = c.host_only;
    a.ncols_dst = static_cast<int32_t>(c.ncols_dst);
    a.nchannels_dst = static_cast<int32_t>(c.nchannels_dst);
    a.n_experts = e->n_experts;
    a.dst = c.dst;
    a.stride_col_dst = c.stride_col_dst;
    a.stride_channel_dst = c.stride_channel_dst;
    a.K = static_cast<int32_t>(c.ne00);
    a.nrows = static_cast<int32_t>(c.ne01);
    a.row_bytes = static_cast<uint32_t>(c.s01 * type_size(src0->type));
    if (a.row_bytes != src0->nb[1]) return fail(MOE_ERR_INVALID, "s01 does not match src0->nb[1]");
    a.err = g.d_err;
    a.timeout_ns = g.timeout_ns_kernel;
    const char *why = "";
    cudaError_t ce = cudaSuccess;
    const int act = c.src1_type == MOE_TYPE_Q8_1 ? moe::ACT_Q8_1 : moe::ACT_CPU;
    rc = moe::launch_gemv(src0->type, act, a, stream, &why, &ce);
    if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
    if (rc) return fail(rc, "%s", why);
    return MOE_OK;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct LayerWs {
    uint32_t *gbar;   // fused kernel: [0] launch epoch, [1] finished CTAs (first 256 bytes)
    int32_t *ids;
    float *w, *h, *hs, *y, *ys;
    float *hg, *hsg;  // gate outputs when gate and up differ in type
    uint64_t *h_tag, *hs_tag;   // fused kernel: h / hs as (value, tag) pairs
    uint32_t *rowcnt;           // per-expert-group kernel: output rows arrived per (token, row block)
    size_t bytes;
};

LayerWs layer_ws(const moe_layer_desc *L, int64_t n_tok, char *base) {
    LayerWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
    const int64_t k = L->k, F = L->F, H = L->H;
    // the epoch sits at offset 0 for every n_tok, so workspaces reused across
    // batch sizes share one tag sequence
    w.gbar = reinterpret_cast<uint32_t *>(take(sizeof(uint32_t) * 2));
    // the row counters follow at a fixed place too, sized for 8 tokens: they
    // are zero between launches whatever batch size used the workspace last
    w.rowcnt = reinterpret_cast<uint32_t *>(take(sizeof(uint32_t) * 8 * ((H + moe::LAYER2_RB - 1) / moe::LAYER2_RB)));
    w.ids = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * n_tok * k));
    w.w = reinterpret_cast<float *>(take(sizeof(float) * n_tok * k));
    w.h = reinterpret_cast<float *>(take(sizeof(float) * n_tok * k * F));
    w.hs = reinterpret_cast<float *>(take(sizeof(float) * n_tok * F));
    w.y = reinterpret_cast<float *>(take(sizeof(float) * n_tok * k * H));
    w.ys = reinterpret_cast<float *>(take(sizeof(float) * n_tok * H));
    w.h_tag = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * n_tok * k * F));
    w.hs_tag = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * n_tok * F));
    w.hg = reinterpret_cast<float *>(take(sizeof(float) * n_tok * k * F));
    w.hsg = reinterpret_cast<float *>(take(sizeof(float) * n_tok * F));
    w.bytes = off;
    return w;
}


// One expert tensor of a fused layer: cache-registered tensors keep their
// bookkeeping; host-tiered ones are read through their table, HBM-resident
// ones at their dense address (what their table holds).
int layer_tensor(const moe_tensor *t, bool registered, cudaStream_t st, moe::LayerTensor *out) {
    *out = moe::LayerTensor{};
    if (registered) {
        Tensor *e = nullptr;
        const int rc = enroll(t, st, &e);
        if (rc) return rc;
        out->stamps = e->stamps;
        out->cache_id = e->id;
        if (e->tiered) out->tbl = e->table;
    }
    out->dense = static_cast<const char *>(t->data);
    out->expert_bytes = t->nb[2];
    out->tma = aligned16(t->data) && (t->nb[2] % 16) == 0 && (out->tbl || ptr_kind(t->data) == 2);
    return MOE_OK;
}

// Fills the fused kernel's arguments for layer L (geometry excluded).
int layer_args(const moe_layer_desc *L, const float *x, const float *logits, float *out, int64_t n_tok,
               const LayerWs &w, cudaStream_t st, moe::LayerArgs *pa) {
    moe::LayerArgs &a = *pa;
    a = moe::LayerArgs{};
    const int64_t k = L->k, F = L->F, H = L->H;
    const bool shared = L->shared_type >= 0;
    if (!aligned16(L->up.data) || !aligned16(L->gate.data) || !aligned16(L->down.data))
        return fail(MOE_ERR_UNSUPPORTED, "expert tensor data must be 16-byte aligned");
    if (shared && (!aligned16(L->shared_up) || !aligned16(L->shared_gate) || !aligned16(L->shared_down)))
        return fail(MOE_ERR_UNSUPPORTED, "gate / shared expert data must be 16-byte aligned");
    int rc = layer_tensor(&L->up, true, st, &a.up);
    if (!rc) rc = layer_tensor(&L->gate, wants_locked(&L->gate) != 0, st, &a.gate);
    if (!rc) rc = layer_tensor(&L->down, true, st, &a.down);
    if (rc) return rc;
    moe::GemvArgs &u = a.gu;
    u.y = x;
    u.stride_col_y = H;
    u.nchannels_y = 1;
    u.ncols_dst = static_cast<int32_t>(n_tok);
    u.nchannels_dst = static_cast<int32_t>(k);
    u.n_experts = static_cast<int32_t>(L->n_experts);
    u.dst = w.h;
    u.stride_col_dst = k * F;
    u.stride_channel_dst = F;
    u.has_fusion = 1;
    u.use_gate = 1;
    u.glu_op = L->glu_op;
    u.glu_limit = L->glu_limit;
    u.K = static_cast<int32_t>(H);
    u.nrows = static_cast<int32_t>(F);
    u.row_bytes = static_cast<uint32_t>(L->up.nb[1]);
    moe::GemvArgs &d = a.dn;
    d.y = w.h;
    d.stride_col_y = k * F;
    d.stride_channel_y = F;
    d.nchannels_y = static_cast<int32_t>(k);
    d.ncols_dst = static_cast<int32_t>(n_tok);
    d.nchannels_dst = static_cast<int32_t>(k);
    d.n_experts = static_cast<int32_t>(L->n_experts);
    d.dst = w.y;
    d.stride_col_dst = k * H;
    d.stride_channel_dst = H;
    d.K = static_cast<int32_t>(F);
    d.nrows = static_cast<int32_t>(H);
    d.row_bytes = static_cast<uint32_t>(L->down.nb[1]);
    if (shared) {
        u.shared_up = static_cast<const char *>(L->shared_up);
        u.shared_gate = static_cast<const char *>(L->shared_gate);
        u.shared_dst = w.hs;
        u.shared_stride_col_dst = F;
        u.tma_shared = (L->up.nb[2] % 16) == 0 && ptr_kind(L->shared_up) == 2 && ptr_kind(L->shared_gate) == 2;
        d.shared_up = static_cast<const char *>(L->shared_down);
        d.shared_dst = w.ys;
        d.shared_stride_col_dst = H;
        d.shared_y = w.hs;
        d.shared_y_stride_col = F;
        a.shared_down = static_cast<const char *>(L->shared_down);
        a.tma_shared_down = (L->down.nb[2] % 16) == 0 && ptr_kind(L->shared_down) == 2;
    }
    a.logits = logits;
    a.n_tok = static_cast<int32_t>(n_tok);
    a.k = static_cast<int32_t>(k);
    a.n_experts = static_cast<int32_t>(L->n_experts);
    a.norm_w = L->norm_w;
    a.ids_out = w.ids;
    a.w_out = w.w;
    a.out = out;
    a.stats = g.d_log;
    a.clock = clock_ptr();
    a.log_cap = kLogCap;
    a.gbar = w.gbar;
    a.h_tag = w.h_tag;
    a.hs_tag = shared ? w.hs_tag : nullptr;
    a.err = g.d_err;
    a.timeout_ns = g.timeout_ns_kernel;
    u.err = d.err = g.d_err;
    u.timeout_ns = d.timeout_ns = g.timeout_ns_kernel;
    return MOE_OK;
}

// The per-expert-group kernel's arguments from the fused-layer fields.
moe::Layer2Args to_layer2(const moe::LayerArgs &a, uint32_t *rowcnt) {
    moe::Layer2Args b{};
    b.gu = a.gu;
    b.dn = a.dn;
    b.up = a.up;
    b.gate = a.gate;
    b.down = a.down;
    b.shared_down = a.shared_down;
    b.tma_shared_down = a.tma_shared_down;
    b.logits = a.logits;
    b.n_tok = a.n_tok;
    b.k = a.k;
    b.n_experts = a.n_experts;
    b.norm_w = a.norm_w;
    b.ids_out = a.ids_out;
    b.w_out = a.w_out;
    b.out = a.out;
    b.stats = a.stats;
    b.clock = a.clock;
    b.log_cap = a.log_cap;
    b.h_tag = a.h_tag;
    b.hs_tag = a.hs_tag;
    b.gbar = a.gbar;
    b.rowcnt = rowcnt;
    b.err = a.err;
    b.timeout_ns = a.timeout_ns;
    return b;
}

// True when the fused kernel takes this layer (type pair, sizes, switch).
bool layer_fusable(const moe_layer_desc *L, int64_t n_tok) {
    if (!g.layer_fused || L->gate.type != L->up.type) return false;
    moe::LayerArgs a{};
    a.n_tok = static_cast<int32_t>(n_tok);
    a.k = static_cast<int32_t>(L->k);
    a.n_experts = static_cast<int32_t>(L->n_experts);
    a.gu.K = static_cast<int32_t>(L->H);
    a.gu.nrows = static_cast<int32_t>(L->F);
    a.gu.row_bytes = static_cast<uint32_t>(L->up.nb[1]);
    a.dn.K = static_cast<int32_t>(L->F);
    a.dn.nrows = static_cast<int32_t>(L->H);
    a.dn.row_bytes = static_cast<uint32_t>(L->down.nb[1]);
    a.gu.shared_up = L->shared_type >= 0 ? static_cast<const char *>(L->shared_up) : nullptr;
    int grid = 0;
    size_t smem = 0;
    const char *why = "";
    if (g.layer_fused == 2) return moe::plan_layer(L->up.type, L->down.type, a, &grid, &smem, &why) == 0;
    moe::Layer2Args b = to_layer2(a, nullptr);
    return moe::plan_layer2(L->up.type, L->down.type, b, &grid, &smem, &why) == 0;
}


// Prefill workspace: the tokens' Q8_K blocks, then the grouping arrays
struct PrefillWs {
    uint8_t *x8, *btiles;
    int32_t *entries, *n_chunks;
    int32_t *pool_ids;             // host-tiered tensors: each pick's pool slot (-1: host memory)
    int4 *chunks;
    int64_t max_chunks;
    size_t bytes;
};

// Tokens per chunk of the tensor-core path (the type's width). Narrower
// chunks do not speed up a one-expert call with few tiles: a tile's cost is
// the per-super-block unpack of its weight rows, which more chunks repeat.
int chunk_tokens_for(const moe_tensor *src0, int64_t) {
    const int ntc = moe::mmq_chunk_tokens(src0->type);
    return ntc > 0 ? ntc : moe::MMQ_NT;
}

// x_rows: activation rows (n_tok, or n_tok * k when each pick has its own row)
PrefillWs prefill_ws(const moe_tensor *src0, int64_t n_tok, int64_t k, int64_t x_rows, char *base) {
    PrefillWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
    const int64_t E = src0->ne[2], K = src0->ne[0];
    // the grouping first: its place depends only on the entries, the experts
    // and the chunk width, so a later call on the same ids can reuse it
    w.entries = reinterpret_cast<int32_t *>(take(4 * n_tok * k));
    w.max_chunks = moe::mmq_max_chunks(n_tok * k, E, chunk_tokens_for(src0, n_tok * k));
    w.chunks = reinterpret_cast<int4 *>(take(16 * static_cast<size_t>(w.max_chunks)));
    w.n_chunks = reinterpret_cast<int32_t *>(take(4));
    w.pool_ids = reinterpret_cast<int32_t *>(take(4 * n_tok * k));
    // activation rows: Q8_K (292 bytes / 256) or, for the 32-weight-block
    // types, Q8_0 (34 bytes / 32); B tiles per (chunk, step)
    const bool b32 = moe::mmq_b32(src0->type);
    w.x8 = reinterpret_cast<uint8_t *>(take(static_cast<size_t>(x_rows) * (b32 ? (K / 32) * 34 : (K / 256) * 292)));
    const int64_t steps = K / (b32 ? moe::mmq_step(src0->type) : 256);
    w.btiles = reinterpret_cast<uint8_t *>(
        take(static_cast<size_t>(w.max_chunks) * steps * (b32 ? moe::mmq_bt_stride(src0->type) : moe::MMQ_BT_BYTES)));
    w.bytes = off;
    return w;
}


// One prefill MUL_MAT_ID: dst[(t * k + p) * rows + r] = row r of expert
// ids[t][p] . x row (t, or t * k + p when x_per_pick). Tensor cores where
// the type and shape allow (grouping, Q8_K quantization, B-tile gather, MMQ),
// else the decode GEMV over chunks of 8 tokens. With dst2 / src2 set (a
// second tensor of the same type and shape, e.g. up beside gate), the second
// product reuses the grouping and the B tiles.
int run_prefill(const moe_tensor *src0, const float *x, bool x_per_pick, int64_t n_tok, const int32_t *ids, int64_t k,
                int64_t ids_stride, float *dst, char *workspace, size_t workspace_bytes, bool *used_tc,
                cudaStream_t st, const moe_tensor *src2 = nullptr, float *dst2 = nullptr, bool ids_zero = false,
                bool reuse_groups = false) {
    *used_tc = false;
    if (!src0 || !src0->data || !x || !ids || !dst) return fail(MOE_ERR_INVALID, "null argument");
    if (n_tok < 1 || k < 1 || ids_stride < k) return fail(MOE_ERR_INVALID, "need n_tok >= 1, k >= 1, ids_stride >= k");
    if (!type_supported(src0->type)) return fail(MOE_ERR_UNSUPPORTED, "unsupported expert type %d", src0->type);
    if (!contiguous(src0) || !aligned16(src0->data))
        return fail(MOE_ERR_UNSUPPORTED, "expert tensor must be contiguous and 16-byte aligned");
    const int64_t K = src0->ne[0], rows = src0->ne[1], E = src0->ne[2];
    const int64_t x_rows = x_per_pick ? n_tok * k : n_tok;
    auto tc_ok = [&](const moe_tensor *t) {
        return moe::mmq_supported(t->type, t->ne[0], t->ne[1]) && ptr_kind(t->data) == 2 && (t->nb[2] % 16) == 0 &&
               contiguous(t) && aligned16(t->data) && n_tok * k < (int64_t{1} << 30) && t->ne[2] <= 16384;
    };
    const bool tc = tc_ok(src0);
    const bool pair = src2 && dst2 && tc && tc_ok(src2) && src2->type == src0->type && src2->ne[0] == K &&
                      src2->ne[1] == rows && src2->ne[2] == E;
    // a host-tiered tensor: the picks of pool-resident experts on the tensor
    // cores (the pool as the expert array, slots as expert ids), the others
    // through the GEMV reading pinned host memory in place
    Tensor *te = nullptr;
    const bool tiered_tc = !tc && !reuse_groups && ptr_kind(src0->data) != 2 &&
                           moe::mmq_supported(src0->type, K, rows) && n_tok * k < (int64_t{1} << 30) &&
                           wants_locked(src0) && enroll(src0, st, &te) == MOE_OK && te && te->tiered && te->pool &&
                           te->n_slots > 0 && te->expert_bytes % 16 == 0 && aligned16(te->pool);
    if (tiered_tc) {
        for (int64_t t0 = 0; t0 < n_tok; t0 += 8) {
            const int64_t nt = n_tok - t0 < 8 ? n_tok - t0 : 8;
            MmvqCall c;
            c.src0 = src0;
            c.src1 = x + t0 * (x_per_pick ? k : 1) * K;
            c.src1_type = MOE_TYPE_F32;
            c.ids = ids + t0 * ids_stride;
            c.dst = dst + t0 * k * rows;
            c.ne00 = K; c.ne01 = rows; c.ncols_dst = nt; c.s01 = static_cast<int64_t>(src0->nb[1]) / type_size(src0->type);
            c.nchannels_y = x_per_pick ? k : 1; c.nchannels_dst = k;
            c.stride_col_y = (x_per_pick ? k : 1) * K; c.stride_channel_y = x_per_pick ? K : 0;
            c.stride_col_dst = k * rows; c.stride_channel_dst = rows;
            c.ids_stride = ids_stride;
            c.host_only = 1;
            const int rc = run_mmvq(c, st);
            if (rc) return rc;
        }
        const PrefillWs w = prefill_ws(src0, n_tok, k, x_rows, workspace);
        if (!workspace || workspace_bytes < w.bytes)
            return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
        int rc = ensure_device();
        if (rc) return rc;
        const int ntc = chunk_tokens_for(src0, n_tok * k);
        CK(moe::launch_mmq_pool_ids(ids, ids_stride, static_cast<int>(n_tok), static_cast<int>(k), te->table,
                                    te->n_experts, te->pool, te->expert_bytes, te->n_slots, w.pool_ids, st));
        CK(moe::launch_mmq_group(w.pool_ids, k, static_cast<int>(n_tok), static_cast<int>(k), te->n_slots, ntc,
                                 w.entries, w.chunks, w.n_chunks, g.d_err, st, true));
        if (moe::mmq_b32(src0->type)) {
            CK(moe::launch_quantize_act(MOE_TYPE_Q8_0, x, w.x8, x_rows, K, st));
            CK(moe::launch_mmq_gather32(w.x8, static_cast<int>(K), moe::mmq_step(src0->type),
                                        x_per_pick ? 1 : static_cast<int>(k), ntc, w.entries, w.chunks, w.n_chunks,
                                        w.max_chunks, w.btiles, moe::mmq_bt_stride(src0->type), st));
        } else {
            CK(moe::launch_quantize_act(MOE_TYPE_Q8_K, x, w.x8, x_rows, K, st));
            CK(moe::launch_mmq_gather(w.x8, static_cast<int>(K), x_per_pick ? 1 : static_cast<int>(k), ntc, w.entries,
                                      w.chunks, w.n_chunks, w.max_chunks, w.btiles, st));
        }
        moe::MmqArgs a{};
        a.dense = te->pool;
        a.expert_bytes = te->expert_bytes;
        a.n_experts = te->n_slots;
        a.K = static_cast<int32_t>(K);
        a.nrows = static_cast<int32_t>(rows);
        a.row_bytes = static_cast<uint32_t>(src0->nb[1]);
        a.btiles = w.btiles;
        a.bt_stride = moe::mmq_bt_stride(src0->type);
        a.n_tok = static_cast<int32_t>(n_tok);
        a.k = static_cast<int32_t>(k);
        a.entries = w.entries;
        a.chunks = w.chunks;
        a.n_chunks = w.n_chunks;
        a.dst = dst;
        a.err = g.d_err;
        a.timeout_ns = g.timeout_ns_kernel;
        const char *why = "";
        cudaError_t ce = cudaSuccess;
        rc = moe::launch_mmq(src0->type, a, st, &why, &ce);
        if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
        if (rc) return fail(rc, "%s", why);
        *used_tc = true;
    } else if (!tc) {
        // no tensor-core path: the decode GEMV over chunks of 8 tokens
        for (int64_t t0 = 0; t0 < n_tok; t0 += 8) {
            const int64_t nt = n_tok - t0 < 8 ? n_tok - t0 : 8;
            MmvqCall c;
            c.src0 = src0;
            c.src1 = x + t0 * (x_per_pick ? k : 1) * K;
            c.src1_type = MOE_TYPE_F32;
            c.ids = ids + t0 * ids_stride;
            c.dst = dst + t0 * k * rows;
            c.ne00 = K; c.ne01 = rows; c.ncols_dst = nt; c.s01 = static_cast<int64_t>(src0->nb[1]) / type_size(src0->type);
            c.nchannels_y = x_per_pick ? k : 1; c.nchannels_dst = k;
            c.stride_col_y = (x_per_pick ? k : 1) * K; c.stride_channel_y = x_per_pick ? K : 0;
            c.stride_col_dst = k * rows; c.stride_channel_dst = rows;
            c.ids_stride = ids_stride;
            const int rc = run_mmvq(c, st);
            if (rc) return rc;
        }
    } else {
        const PrefillWs w = prefill_ws(src0, n_tok, k, x_rows, workspace);
        if (!workspace || workspace_bytes < w.bytes)
            return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
        int rc = ensure_device();
        if (rc) return rc;
        const int ntc = chunk_tokens_for(src0, n_tok * k);
        if (reuse_groups) {
            // the previous call on this workspace grouped the same ids over the
            // same experts with the same chunk width
        } else if (ids_zero && E == 1 && k == 1)   // the caller's ids are all 0: entries in order
            CK(moe::launch_mmq_identity_chunks(static_cast<int>(n_tok), ntc, w.entries, w.chunks, w.n_chunks, st));
        else
            CK(moe::launch_mmq_group(ids, ids_stride, static_cast<int>(n_tok), static_cast<int>(k), static_cast<int>(E),
                                     ntc, w.entries, w.chunks, w.n_chunks, g.d_err, st));
        // the gather reads activation row entry / k_div (entry = t * k + p)
        if (moe::mmq_b32(src0->type)) {
            CK(moe::launch_quantize_act(MOE_TYPE_Q8_0, x, w.x8, x_rows, K, st));
            CK(moe::launch_mmq_gather32(w.x8, static_cast<int>(K), moe::mmq_step(src0->type),
                                        x_per_pick ? 1 : static_cast<int>(k), ntc, w.entries, w.chunks, w.n_chunks,
                                        w.max_chunks, w.btiles, moe::mmq_bt_stride(src0->type), st));
        } else {
            CK(moe::launch_quantize_act(MOE_TYPE_Q8_K, x, w.x8, x_rows, K, st));
            CK(moe::launch_mmq_gather(w.x8, static_cast<int>(K), x_per_pick ? 1 : static_cast<int>(k), ntc, w.entries,
                                      w.chunks, w.n_chunks, w.max_chunks, w.btiles, st));
        }
        for (int pass = 0; pass < (pair ? 2 : 1); ++pass) {
            const moe_tensor *t = pass == 0 ? src0 : src2;
            moe::MmqArgs a{};
            a.dense = static_cast<const char *>(t->data);
            a.expert_bytes = t->nb[2];
            a.n_experts = static_cast<int32_t>(E);
            a.K = static_cast<int32_t>(K);
            a.nrows = static_cast<int32_t>(rows);
            a.row_bytes = static_cast<uint32_t>(t->nb[1]);
            a.btiles = w.btiles;
            a.bt_stride = moe::mmq_bt_stride(t->type);
            a.n_tok = static_cast<int32_t>(n_tok);
            a.k = static_cast<int32_t>(k);
            a.entries = w.entries;
            a.chunks = w.chunks;
            a.n_chunks = w.n_chunks;
            a.dst = pass == 0 ? dst : dst2;
            a.err = g.d_err;
            a.timeout_ns = g.timeout_ns_kernel;
            const char *why = "";
            cudaError_t ce = cudaSuccess;
            rc = moe::launch_mmq(t->type, a, st, &why, &ce);
            if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
            if (rc) return fail(rc, "%s", why);
        }
        *used_tc = true;
    }
    if (src2 && dst2 && !pair) {   // the second tensor on its own
        bool tc2 = false;
        return run_prefill(src2, x, x_per_pick, n_tok, ids, k, ids_stride, dst2, workspace, workspace_bytes, &tc2, st);
    }
    return MOE_OK;
}

// A shared-expert matrix as a one-expert tensor of the given type
moe_tensor shared_tensor(const void *data, int32_t type, int64_t K, int64_t rows) {
    moe_tensor t{};
    t.data = const_cast<void *>(data);
    t.type = type;
    const uint64_t rb = static_cast<uint64_t>(K / blck_size(type)) * type_size(type);
    t.ne[0] = K; t.ne[1] = rows; t.ne[2] = 1; t.ne[3] = 1;
    t.nb[0] = type_size(type); t.nb[1] = rb; t.nb[2] = rb * rows; t.nb[3] = rb * rows;
    return t;
}

// Layer prefill workspace: ids, weights, gate / up (then h) / down outputs,
// the shared expert's outputs, zero ids, then the MUL_MAT_ID scratch
struct LayerPrefillWs {
    int32_t *ids, *zero_ids;
    float *w, *g, *u, *y, *sg, *su, *ys;
    char *scratch;
    size_t scratch_bytes, bytes;
};

// k picks per token (the layer's k, or 1 for expert-parallel received rows)
LayerPrefillWs layer_prefill_ws(const moe_layer_desc *L, int64_t n, int64_t k, char *base) {
    LayerPrefillWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
    const int64_t H = L->H, F = L->F;
    w.ids = reinterpret_cast<int32_t *>(take(4 * n * k));
    w.w = reinterpret_cast<float *>(take(4 * n * k));
    w.g = reinterpret_cast<float *>(take(4 * n * k * F));
    w.u = reinterpret_cast<float *>(take(4 * n * k * F));
    w.y = reinterpret_cast<float *>(take(4 * n * k * H));
    const bool shared = L->shared_type >= 0;
    if (shared) {
        w.sg = reinterpret_cast<float *>(take(4 * n * F));
        w.su = reinterpret_cast<float *>(take(4 * n * F));
        w.ys = reinterpret_cast<float *>(take(4 * n * H));
        w.zero_ids = reinterpret_cast<int32_t *>(take(4 * n));
    }
    size_t sc = 0;
    auto need = [&](const moe_tensor &t, int64_t kk, int64_t rows) {
        const size_t b = prefill_ws(&t, n, kk, rows, nullptr).bytes;
        sc = b > sc ? b : sc;
    };
    need(L->gate, k, n * k);   // rows: per pick when the caller gives one row per pick
    need(L->up, k, n * k);
    need(L->down, k, n * k);
    if (shared) {
        const moe_tensor sg = shared_tensor(L->shared_gate, L->gate.type, H, F);
        const moe_tensor su = shared_tensor(L->shared_up, L->up.type, H, F);
        const moe_tensor sd = shared_tensor(L->shared_down, L->down.type, F, H);
        need(sg, 1, n);
        need(su, 1, n);
        need(sd, 1, n);
    }
    w.scratch = take(sc);
    w.scratch_bytes = sc;
    w.bytes = off;
    return w;
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

int ggml_cuda_moe_cache_enabled(void) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    return g.enabled ? 1 : 0;
}

int ggml_cuda_moe_cache_wants(const moe_tensor *src0) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return wants_locked(src0);
}

int ggml_cuda_moe_cache_mul_mat_vec_q(const moe_tensor *src0, const moe_fusion_host *fusion,
                                      const moe_fusion_device *fusion_dev, const void *src1, int32_t src1_type,
                                      const int32_t *ids_d, float *dst_d, int64_t ne00, int64_t ne01, int64_t ne02,
                                      int64_t ne03, int64_t ncols_dst, int64_t s01, int64_t s02, int64_t s03,
                                      int64_t nchannels_y, int64_t nchannels_dst, int64_t stride_col_y,
                                      int64_t stride_col_dst, int64_t stride_channel_y, int64_t stride_channel_dst,
                                      int64_t ids_stride, moe_stream_t stream) {
    (void)ne02; (void)ne03; (void)s02; (void)s03;
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    MmvqCall c;
    c.src0 = src0;
    c.gate = fusion ? fusion->gate : nullptr;
    c.fd = fusion_dev;
    c.src1 = src1;
    c.src1_type = src1_type;
    c.ids = ids_d;
    c.dst = dst_d;
    c.ne00 = ne00; c.ne01 = ne01; c.ncols_dst = ncols_dst; c.s01 = s01;
    c.nchannels_y = nchannels_y; c.nchannels_dst = nchannels_dst;
    c.stride_col_y = stride_col_y; c.stride_col_dst = stride_col_dst;
    c.stride_channel_y = stride_channel_y; c.stride_channel_dst = stride_channel_dst;
    c.ids_stride = ids_stride;
    return run_mmvq(c, reinterpret_cast<cudaStream_t>(stream));
}

int ggml_cuda_moe_cache_step(moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return step_locked(reinterpret_cast<cudaStream_t>(stream));
}

int ggml_cuda_moe_cache_active(void) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return g.tensors.empty() ? 0 : 1;
}

// reference ggml_cuda_moe_cache_pin_host (:372-405)
int ggml_cuda_moe_cache_pin_host(const moe_tensor *t) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!g.enabled || !t || (t->flags & MOE_TENSOR_NO_BUFFER) || !t->data) return 0;
    cudaPointerAttributes attrs;
    cudaError_t err = cudaPointerGetAttributes(&attrs, t->data);
    if (err != cudaSuccess) { cudaGetLastError(); return 0; }
    if (attrs.type == cudaMemoryTypeHost || attrs.type == cudaMemoryTypeManaged) return 1;
    if (attrs.type == cudaMemoryTypeDevice) return 0;
    const int64_t bs = blck_size(t->type);
    uint64_t nbytes = static_cast<uint64_t>(t->ne[0] / bs) * t->nb[0];
    for (int i = 1; i < 4; ++i) nbytes += static_cast<uint64_t>(t->ne[i] - 1) * t->nb[i];
    const uintptr_t page = 4096;
    const uintptr_t base = reinterpret_cast<uintptr_t>(t->data) & ~(page - 1);
    const uintptr_t end = (reinterpret_cast<uintptr_t>(t->data) + nbytes + page - 1) & ~(page - 1);
    err = cudaHostRegister(reinterpret_cast<void *>(base), end - base, cudaHostRegisterPortable | cudaHostRegisterReadOnly);
    if (err == cudaSuccess) {
        g.ptr_kind.erase(t->data);
        return 1;
    }
    cudaGetLastError();
    fail(MOE_ERR_CUDA, "moe-cache: failed to pin %s: %s", t->name ? t->name : "<tensor>", cudaGetErrorString(err));
    return 0;
}

int moe_b200_configure(const moe_cache_config *cfg) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!cfg) return fail(MOE_ERR_INVALID, "null config");
    free_all();
    g.enabled = cfg->enabled != 0;
    g.slots = cfg->slots < 0 ? 0 : cfg->slots;
    g.budget = cfg->budget_gb > 0 ? static_cast<size_t>(cfg->budget_gb * 1024.0 * 1024.0 * 1024.0) : (30ull << 30);
    g.seed_path = cfg->seed_path ? cfg->seed_path : "";
    g.claim_device = cfg->claim_device != 0;
    g.debug = cfg->debug != 0;
    g.env_read = true;
    g.configured = true;
    // the kernel choice is not cache configuration: the environment still picks it
    g.layer_fused = std::min(2, std::max(0, env_int("GGML_CUDA_MOE_LAYER_FUSED", g.layer_fused)));
    return MOE_OK;
}

int moe_b200_reset(void) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    free_all();
    g.env_read = false;
    g.configured = false;
    g.enabled = false;
    g.slots = 320;
    g.budget = 30ull << 30;
    g.claim_device = true;
    g.debug = false;
    g.seed_path.clear();
    return MOE_OK;
}

int moe_b200_stats(moe_cache_stats *out) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!out) return fail(MOE_ERR_INVALID, "null stats");
    memset(out, 0, sizeof(*out));
    out->registered = g.tensors.size();
    out->pool_bytes = g.pool_bytes;
    out->steps = g.idle_steps;
    if (!g.dev) return MOE_OK;
    // totals live on the device (the promotion pass keeps them)
    moe::CacheDev s;
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(&s, g.dev, sizeof(s), cudaMemcpyDeviceToHost));
    out->steps += s.steps;
    out->hits = s.hits;
    out->misses = s.misses;
    out->promotions = s.promotions;
    out->evictions = s.evictions;
    out->log_overflow = s.overflow;
    for (const Tensor *t : g.tensors) {
        if (t->retired || t->n_slots == 0) continue;
        std::vector<int32_t> owner(static_cast<size_t>(t->n_slots));
        CK(cudaMemcpy(owner.data(), t->slot_owner, 4 * owner.size(), cudaMemcpyDeviceToHost));
        for (const int32_t x : owner) out->resident += x >= 0;
    }
    return MOE_OK;
}

int moe_b200_table(const void *data, int32_t *slot_of, int32_t n_experts, int32_t *n_slots, int32_t *tensor_id) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    auto it = g.by_ptr.find(static_cast<const char *>(data));
    if (it == g.by_ptr.end()) return fail(MOE_ERR_INVALID, "tensor is not registered");
    const Tensor *t = it->second;
    if (n_experts < t->n_experts) return fail(MOE_ERR_INVALID, "slot_of too small");
    std::vector<char *> tbl(t->n_experts);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(tbl.data(), t->table, sizeof(char *) * t->n_experts, cudaMemcpyDeviceToHost));
    const uintptr_t pool = reinterpret_cast<uintptr_t>(t->pool);
    const uintptr_t pool_end = pool + static_cast<uintptr_t>(t->n_slots) * t->expert_bytes;
    for (int i = 0; i < t->n_experts; ++i) {
        const uintptr_t p = reinterpret_cast<uintptr_t>(tbl[i]);
        if (p & 1u) slot_of[i] = -1;
        else if (t->pool && p >= pool && p < pool_end) slot_of[i] = static_cast<int32_t>((p - pool) / t->expert_bytes);
        else slot_of[i] = -2;
    }
    if (n_slots) *n_slots = t->n_slots;
    if (tensor_id) *tensor_id = t->id;
    return MOE_OK;
}

int moe_b200_device_error(moe_stream_t stream, int32_t *code) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (code) *code = 0;
    CK(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
    if (!g.d_err) return MOE_OK;
    int v = 0;
    CK(cudaMemcpy(&v, g.d_err, sizeof(int), cudaMemcpyDeviceToHost));
    CK(cudaMemset(g.d_err, 0, sizeof(int)));
    if (code) *code = v;
    return MOE_OK;
}

const char *moe_b200_last_error(void) { return g_err.c_str(); }

int moe_b200_quantize_act(int32_t act_type, const float *x, void *y, int64_t n_rows, int64_t n_cols, moe_stream_t stream) {
    if (act_type != MOE_TYPE_Q8_0 && act_type != MOE_TYPE_Q8_1 && act_type != MOE_TYPE_Q8_K)
        return fail(MOE_ERR_UNSUPPORTED, "act_type must be Q8_0, Q8_1 or Q8_K");
    const int64_t qk = act_type == MOE_TYPE_Q8_K ? 256 : 32;
    if (n_cols % qk || n_rows < 0) return fail(MOE_ERR_INVALID, "n_cols must be a multiple of %lld", static_cast<long long>(qk));
    CK(moe::launch_quantize_act(act_type, x, y, n_rows, n_cols, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

int moe_b200_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts, int64_t k, int32_t norm_w, int32_t *ids,
                          float *weights, moe_stream_t stream) {
    if (k < 1 || k > 32 || k > n_experts || n_experts > 65536) return fail(MOE_ERR_INVALID, "need 1 <= k <= min(32, n_experts)");
    CK(moe::launch_topk_softmax(logits, n_tok, n_experts, k, norm_w, ids, weights, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

size_t moe_b200_layer_workspace_size(const moe_layer_desc *L, int64_t n_tok) {
    if (!L) return 0;
    return layer_ws(L, n_tok, nullptr).bytes;
}

int moe_b200_layer_decode(const moe_layer_desc *L, const float *x, const float *logits, float *out, int64_t n_tok,
                          void *workspace, size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !logits || !out) return fail(MOE_ERR_INVALID, "null argument");
    if (n_tok < 1 || n_tok > 8) return fail(MOE_ERR_UNSUPPORTED, "layer decode handles 1..8 tokens");
    const LayerWs w = layer_ws(L, n_tok, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes) return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu)", workspace_bytes, w.bytes);
    const bool shared = L->shared_type >= 0;   // the shared gate/up/down take gate's/up's/down's types
    const bool split_gate = L->gate.type != L->up.type;   // no fused gate/up GEMV: two GEMVs and a GLU pass
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t k = L->k, F = L->F, H = L->H;
    if (L->up.ne[0] != H || L->up.ne[1] != F || L->down.ne[0] != F || L->down.ne[1] != H)
        return fail(MOE_ERR_INVALID, "expert tensor shapes do not match H/F");
    if (layer_fusable(L, n_tok)) {
        moe::LayerArgs a;
        int rc = layer_args(L, x, logits, out, n_tok, w, st, &a);
        if (rc) return rc;
        const char *why = "";
        cudaError_t ce = cudaSuccess;
        if (g.layer_fused == 2) {
            rc = moe::launch_layer(L->up.type, L->down.type, a, st, &why, &ce);
        } else {
            moe::Layer2Args b = to_layer2(a, w.rowcnt);
            rc = moe::launch_layer2(L->up.type, L->down.type, b, st, &why, &ce);
        }
        if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
        if (rc) return fail(rc, "%s", why);
        return MOE_OK;
    }
    CK(moe::launch_topk_softmax(logits, n_tok, L->n_experts, k, L->norm_w, w.ids, w.w, st));

    // gate/up: one fused GEMV with the GLU in its epilogue, or (types differ,
    // as llama.cpp then runs them) an up GEMV, a gate GEMV and a GLU pass
    MmvqCall c;
    moe_fusion_device fd{};
    c.src0 = &L->up;
    c.fd = &fd;
    c.src1 = x;
    c.src1_type = MOE_TYPE_F32;
    c.ids = w.ids;
    c.dst = w.h;
    c.ne00 = H; c.ne01 = F; c.ncols_dst = n_tok; c.s01 = static_cast<int64_t>(L->up.nb[1]) / type_size(L->up.type);
    c.nchannels_y = 1; c.nchannels_dst = k;
    c.stride_col_y = H; c.stride_channel_y = 0;
    c.stride_col_dst = k * F; c.stride_channel_dst = F;
    c.ids_stride = k;
    if (shared) {
        fd.shared_up = L->shared_up;
        fd.shared_dst = w.hs;
        fd.shared_stride_col_dst = F;
    }
    int rc;
    if (!split_gate) {
        c.gate = &L->gate;
        fd.gate = L->gate.data;
        fd.glu_op = L->glu_op;
        fd.glu_limit = L->glu_limit;
        if (shared) fd.shared_gate = L->shared_gate;
        rc = run_mmvq(c, st);
        if (rc) return rc;
    } else {
        rc = run_mmvq(c, st);   // up (and the shared up) -> h, hs
        if (rc) return rc;
        MmvqCall cg = c;
        moe_fusion_device fg{};
        cg.src0 = &L->gate;
        cg.fd = &fg;
        cg.dst = w.hg;
        cg.s01 = static_cast<int64_t>(L->gate.nb[1]) / type_size(L->gate.type);
        if (shared) {
            fg.shared_up = L->shared_gate;
            fg.shared_dst = w.hsg;
            fg.shared_stride_col_dst = F;
        }
        rc = run_mmvq(cg, st);   // gate (and the shared gate) -> hg, hsg
        if (rc) return rc;
        CK(moe::launch_glu(w.hg, w.h, n_tok * k * F, L->glu_op, L->glu_limit, st));
        if (shared) CK(moe::launch_glu(w.hsg, w.hs, n_tok * F, L->glu_op, L->glu_limit, st));
    }

    moe_fusion_device fd2{};
    if (shared) {
        fd2.shared_up = L->shared_down;
        fd2.shared_dst = w.ys;
        fd2.shared_stride_col_dst = H;
    }
    MmvqCall d;
    d.src0 = &L->down;
    d.fd = &fd2;
    d.src1 = w.h;
    d.src1_type = MOE_TYPE_F32;
    d.ids = w.ids;
    d.dst = w.y;
    d.ne00 = F; d.ne01 = H; d.ncols_dst = n_tok; d.s01 = static_cast<int64_t>(L->down.nb[1]) / type_size(L->down.type);
    d.nchannels_y = k; d.nchannels_dst = k;
    d.stride_col_y = k * F; d.stride_channel_y = F;
    d.stride_col_dst = k * H; d.stride_channel_dst = H;
    d.ids_stride = k;
    d.shared_y = shared ? w.hs : nullptr;
    d.shared_y_stride_col = F;
    rc = run_mmvq(d, st);
    if (rc) return rc;
    CK(moe::launch_combine(w.y, w.w, shared ? w.ys : nullptr, out, n_tok, H, k, st));
    return MOE_OK;
}

int moe_b200_ep_layer_decode(const moe_layer_desc *L, int64_t expert_lo, int64_t n_experts_global,
                              int32_t with_shared, const float *x, const float *logits, float *out, int64_t n_tok,
                              void *workspace, size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !logits || !out) return fail(MOE_ERR_INVALID, "null argument");
    if (n_tok < 1 || n_tok > 8) return fail(MOE_ERR_UNSUPPORTED, "layer decode handles 1..8 tokens");
    if (expert_lo < 0 || expert_lo + L->n_experts > n_experts_global || n_experts_global > 65536)
        return fail(MOE_ERR_INVALID, "local experts [%lld, %lld) outside the %lld routed experts",
                    static_cast<long long>(expert_lo), static_cast<long long>(expert_lo + L->n_experts),
                    static_cast<long long>(n_experts_global));
    const LayerWs w = layer_ws(L, n_tok, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes) return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu)", workspace_bytes, w.bytes);
    if (L->gate.type != L->up.type) return fail(MOE_ERR_UNSUPPORTED, "expert-parallel decode needs one gate/up type");
    const bool shared = with_shared && L->shared_type >= 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t k = L->k, F = L->F, H = L->H;
    if (k < 1 || k > 32 || k > n_experts_global) return fail(MOE_ERR_INVALID, "need 1 <= k <= min(32, n_experts)");
    if (L->up.ne[0] != H || L->up.ne[1] != F || L->down.ne[0] != F || L->down.ne[1] != H)
        return fail(MOE_ERR_INVALID, "expert tensor shapes do not match H/F");
    // every GPU routes over all experts (same logits, same bits)
    CK(moe::launch_topk_softmax(logits, n_tok, n_experts_global, k, L->norm_w, w.ids, w.w, st));
    moe_fusion_device fd{};
    fd.gate = L->gate.data;
    fd.glu_op = L->glu_op;
    fd.glu_limit = L->glu_limit;
    if (shared) {
        fd.shared_up = L->shared_up;
        fd.shared_gate = L->shared_gate;
        fd.shared_dst = w.hs;
        fd.shared_stride_col_dst = F;
    }
    MmvqCall c;
    c.src0 = &L->up;
    c.gate = &L->gate;
    c.fd = &fd;
    c.src1 = x;
    c.src1_type = MOE_TYPE_F32;
    c.ids = w.ids;
    c.dst = w.h;
    c.ne00 = H; c.ne01 = F; c.ncols_dst = n_tok; c.s01 = static_cast<int64_t>(L->up.nb[1]) / type_size(L->up.type);
    c.nchannels_y = 1; c.nchannels_dst = k;
    c.stride_col_y = H; c.stride_channel_y = 0;
    c.stride_col_dst = k * F; c.stride_channel_dst = F;
    c.ids_stride = k;
    c.id_offset = expert_lo;
    c.skip_foreign = 1;
    int rc = run_mmvq(c, st);
    if (rc) return rc;
    moe_fusion_device fd2{};
    if (shared) {
        fd2.shared_up = L->shared_down;
        fd2.shared_dst = w.ys;
        fd2.shared_stride_col_dst = H;
    }
    MmvqCall d;
    d.src0 = &L->down;
    d.fd = &fd2;
    d.src1 = w.h;
    d.src1_type = MOE_TYPE_F32;
    d.ids = w.ids;
    d.dst = w.y;
    d.ne00 = F; d.ne01 = H; d.ncols_dst = n_tok; d.s01 = static_cast<int64_t>(L->down.nb[1]) / type_size(L->down.type);
    d.nchannels_y = k; d.nchannels_dst = k;
    d.stride_col_y = k * F; d.stride_channel_y = F;
    d.stride_col_dst = k * H; d.stride_channel_dst = H;
    d.ids_stride = k;
    d.shared_y = shared ? w.hs : nullptr;
    d.shared_y_stride_col = F;
    d.id_offset = expert_lo;
    d.skip_foreign = 1;
    rc = run_mmvq(d, st);
    if (rc) return rc;
    // this GPU's share of the weighted sum: its own picks (pick order) and,
    // where it holds it, the shared expert; the caller sums the GPUs' shares
    CK(moe::launch_combine_local(w.y, w.w, shared ? w.ys : nullptr, w.ids, static_cast<int>(expert_lo),
                                 static_cast<int>(L->n_experts), out, n_tok, H, k, st));
    return MOE_OK;
}

size_t moe_b200_prefill_workspace_size(const moe_tensor *src0, int64_t n_tok, int64_t k) {
    if (!src0 || n_tok < 0 || k < 0) return 0;
    return prefill_ws(src0, n_tok, k, n_tok, nullptr).bytes;
}

int moe_b200_prefill_mul_mat_id(const moe_tensor *src0, const float *x, int64_t n_tok, const int32_t *ids, int64_t k,
                                int64_t ids_stride, float *dst, void *workspace, size_t workspace_bytes,
                                int32_t *used_tensor_cores, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    bool tc = false;
    const int rc = run_prefill(src0, x, false, n_tok, ids, k, ids_stride, dst, static_cast<char *>(workspace),
                               workspace_bytes, &tc, reinterpret_cast<cudaStream_t>(stream));
    if (used_tensor_cores) *used_tensor_cores = tc ? 1 : 0;
    return rc;
}

size_t moe_b200_layer_prefill_workspace_size(const moe_layer_desc *L, int64_t n_tok) {
    if (!L || n_tok < 1) return 0;
    return layer_prefill_ws(L, n_tok, L->k, nullptr).bytes;
}

namespace {

// gate and up per pick, GLU, down per pick into y [n][k][H]
int experts_prefill(const moe_layer_desc *L, const float *x, bool x_per_pick, const int32_t *ids, int64_t n_tok,
                    int64_t k, const LayerPrefillWs &w, float *y, cudaStream_t st) {
    bool tc = false;
    // gate and up: one grouping and B-tile gather when they share a type
    int rc = run_prefill(&L->gate, x, x_per_pick, n_tok, ids, k, k, w.g, w.scratch, w.scratch_bytes, &tc, st, &L->up,
                         w.u);
    if (rc) return rc;
    CK(moe::launch_glu(w.g, w.u, n_tok * k * L->F, L->glu_op, L->glu_limit, st));
    // down: same ids and experts; its grouping is the gate/up one when both
    // ran on the tensor cores with the same chunk width
    bool tc_down = false;
    const bool reuse = tc && moe::mmq_supported(L->down.type, L->down.ne[0], L->down.ne[1]) &&
                       ptr_kind(L->down.data) == 2 && (L->down.nb[2] % 16) == 0 &&
                       chunk_tokens_for(&L->down, n_tok * k) == chunk_tokens_for(&L->gate, n_tok * k) &&
                       L->down.ne[2] == L->gate.ne[2] && L->gate.type == L->up.type;
    return run_prefill(&L->down, w.u, true, n_tok, ids, k, k, y, w.scratch, w.scratch_bytes, &tc_down, st, nullptr,
                       nullptr, false, reuse);
}

// the shared expert of every token into ys [n][H]
int shared_prefill(const moe_layer_desc *L, const float *x, int64_t n_tok, const LayerPrefillWs &w, float *ys,
                   cudaStream_t st) {
    const int64_t H = L->H, F = L->F;
    bool tc = false;
    const moe_tensor sg = shared_tensor(L->shared_gate, L->gate.type, H, F);
    const moe_tensor su = shared_tensor(L->shared_up, L->up.type, H, F);
    const moe_tensor sd = shared_tensor(L->shared_down, L->down.type, F, H);
    CK(cudaMemsetAsync(w.zero_ids, 0, 4 * n_tok, st));
    int rc = run_prefill(&sg, x, false, n_tok, w.zero_ids, 1, 1, w.sg, w.scratch, w.scratch_bytes, &tc, st, &su, w.su,
                         true);
    if (rc) return rc;
    CK(moe::launch_glu(w.sg, w.su, n_tok * F, L->glu_op, L->glu_limit, st));
    return run_prefill(&sd, w.su, false, n_tok, w.zero_ids, 1, 1, ys, w.scratch, w.scratch_bytes, &tc, st, nullptr,
                       nullptr, true);   // (the identity table is one cheap launch)
}

}  // namespace

int moe_b200_layer_prefill(const moe_layer_desc *L, const float *x, const float *logits, float *out, int64_t n_tok,
                           void *workspace, size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !logits || !out || n_tok < 1) return fail(MOE_ERR_INVALID, "null argument or n_tok < 1");
    if (L->k < 1 || L->k > L->n_experts || L->k > 32) return fail(MOE_ERR_INVALID, "need 1 <= k <= min(32, n_experts)");
    const LayerPrefillWs w = layer_prefill_ws(L, n_tok, L->k, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes)
        return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    CK(moe::launch_topk_softmax(logits, n_tok, L->n_experts, L->k, L->norm_w, w.ids, w.w, st));
    int rc = experts_prefill(L, x, false, w.ids, n_tok, L->k, w, w.y, st);
    if (rc) return rc;
    if (L->shared_type >= 0) {
        rc = shared_prefill(L, x, n_tok, w, w.ys, st);
        if (rc) return rc;
    }
    CK(moe::launch_combine(w.y, w.w, L->shared_type >= 0 ? w.ys : nullptr, out, n_tok, L->H, L->k, st));
    return MOE_OK;
}

size_t moe_b200_experts_prefill_workspace_size(const moe_layer_desc *L, int64_t n_tok, int64_t k) {
    if (!L || n_tok < 1 || k < 1) return 0;
    return layer_prefill_ws(L, n_tok, k, nullptr).bytes;
}

int moe_b200_experts_prefill(const moe_layer_desc *L, const float *x, int32_t x_per_pick, const int32_t *ids,
                             int64_t n_tok, int64_t k, float *y, void *workspace, size_t workspace_bytes,
                             moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !ids || !y || n_tok < 1 || k < 1) return fail(MOE_ERR_INVALID, "null argument, n_tok < 1 or k < 1");
    const LayerPrefillWs w = layer_prefill_ws(L, n_tok, k, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes)
        return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
    return experts_prefill(L, x, x_per_pick != 0, ids, n_tok, k, w, y, reinterpret_cast<cudaStream_t>(stream));
}

int moe_b200_shared_prefill(const moe_layer_desc *L, const float *x, int64_t n_tok, float *ys, void *workspace,
                            size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !ys || n_tok < 1) return fail(MOE_ERR_INVALID, "null argument or n_tok < 1");
    if (L->shared_type < 0) return fail(MOE_ERR_INVALID, "layer has no shared expert");
    const LayerPrefillWs w = layer_prefill_ws(L, n_tok, L->k, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes)
        return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
    return shared_prefill(L, x, n_tok, w, ys, reinterpret_cast<cudaStream_t>(stream));
}

int moe_b200_combine(const float *y, const float *weights, const float *ys, float *out, int64_t n_tok, int64_t H,
                     int64_t k, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!y || !weights || !out || n_tok < 1 || H < 1 || k < 1) return fail(MOE_ERR_INVALID, "bad combine arguments");
    CK(moe::launch_combine(y, weights, ys, out, n_tok, H, k, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

// ---- expert-parallel exchange over peer memory ------------------------------

}  // extern "C"
namespace {
// rows of the peer table (x: row 0, y_ret: row 3) are copied as float4
bool peer_rows_aligned(const void *const *peer_ptrs, int32_t world) {
    for (int32_t r = 0; r < world; ++r)
        if (!aligned16(peer_ptrs[0 * world + r]) || !aligned16(peer_ptrs[3 * world + r])) return false;
    return true;
}
}  // namespace
extern "C" {

int moe_b200_ipc_alloc(size_t bytes, void **ptr) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!ptr || bytes == 0) return fail(MOE_ERR_INVALID, "null pointer or zero size");
    *ptr = nullptr;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(MOE_ERR_OOM, "cudaMalloc of %zu bytes failed", bytes);
    }
    CK(cudaMemset(*ptr, 0, bytes));
    return MOE_OK;
}

int moe_b200_ipc_free(void *ptr) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (ptr) CK(cudaFree(ptr));
    return MOE_OK;
}

int moe_b200_ipc_handle(const void *ptr, void *handle) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!ptr || !handle) return fail(MOE_ERR_INVALID, "null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == MOE_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)));
    memcpy(handle, &h, sizeof(h));
    return MOE_OK;
}

int moe_b200_ipc_open(const void *handle, void **ptr) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!handle || !ptr) return fail(MOE_ERR_INVALID, "null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    CK(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return MOE_OK;
}

int moe_b200_ipc_close(void *ptr) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (ptr) CK(cudaIpcCloseMemHandle(ptr));
    return MOE_OK;
}

int moe_b200_ep_dispatch(const void *const *peer_ptrs, int32_t world, int32_t rank, int64_t cap, const int32_t *ids,
                         int64_t n_entries, int64_t k, int64_t n_experts, const float *x, int64_t H, void *scratch,
                         moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!peer_ptrs || !ids || !x || !scratch || world < 1 || world > 8 || rank < 0 || rank >= world || k < 1 ||
        n_entries < 0 || n_entries > cap || H % 4 || cap >= (int64_t{1} << 31) / world)
        return fail(MOE_ERR_INVALID, "bad expert-parallel dispatch arguments");
    int rc = ensure_device();
    if (rc) return rc;
    if (!aligned16(x) || !peer_rows_aligned(peer_ptrs, world))
        return fail(MOE_ERR_INVALID, "x and every peer's row buffers (x, y_ret) must be 16-byte aligned");
    CK(moe::launch_ep_dispatch(peer_ptrs, world, rank, static_cast<int>(cap), ids, static_cast<int>(n_entries),
                               static_cast<int>(k), static_cast<int>(n_experts), x, static_cast<int>(H),
                               static_cast<uint32_t *>(scratch), g.d_err, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

int moe_b200_ep_return(const void *const *peer_ptrs, int32_t world, int64_t cap, const int32_t *ids,
                       const int32_t *src, const float *y, int64_t H, void *scratch, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!peer_ptrs || !ids || !src || !y || !scratch || world < 1 || world > 8 || H % 4)
        return fail(MOE_ERR_INVALID, "bad expert-parallel return arguments");
    if (!aligned16(y) || !peer_rows_aligned(peer_ptrs, world))
        return fail(MOE_ERR_INVALID, "y and every peer's row buffers (x, y_ret) must be 16-byte aligned");
    CK(moe::launch_ep_return(peer_ptrs, world, static_cast<int>(cap), ids, src, y, static_cast<int>(H),
                             static_cast<uint32_t *>(scratch), reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

// The stack's workspace: the layer workspace at one token, the layer
// descriptors, then the tagged down rows ([k][H] routed + [H] shared) and the
// tagged x buffers ([2][H]) through which consecutive layers hand over.
struct StackWs {
    moe::StackLayer *layers;
    uint64_t *ytag, *xtag;
    size_t bytes;
};

StackWs stack_ws(const moe_layer_desc *L, int64_t n_layers, char *base) {
    StackWs w{};
    size_t off = layer_ws(L, 1, nullptr).bytes;
    auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
    w.layers = reinterpret_cast<moe::StackLayer *>(take(sizeof(moe::StackLayer) * static_cast<size_t>(n_layers)));
    w.ytag = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * static_cast<size_t>((L->k + 1) * L->H)));
    w.xtag = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * static_cast<size_t>(2 * L->H)));
    w.bytes = off;
    return w;
}

// Mixed stacks: the type slots in use (gate/up, down) of each workspace that
// moe_b200_stack_prepare set up with layers of different types; the launch
// sizes its stages for them. A workspace prepared for one type has no entry.
std::unordered_map<const void *, std::pair<unsigned, unsigned>> g_stack_mixed;

size_t moe_b200_stack_workspace_size(const moe_layer_desc *L, int64_t n_layers) {
    if (!L || n_layers < 1) return 0;
    return stack_ws(L, n_layers, nullptr).bytes;
}

int moe_b200_stack_prepare(const moe_layer_desc *layers, int64_t n_layers, const float *const *x,
                           const float *const *logits, float *const *out, float *const *x_next, void *workspace,
                           size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!layers || n_layers < 1 || !x || !logits || !out) return fail(MOE_ERR_INVALID, "null argument");
    const moe_layer_desc &L0 = layers[0];
    const size_t need = moe_b200_stack_workspace_size(&L0, n_layers);
    if (!workspace || workspace_bytes < need) return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu)", workspace_bytes, need);
    // one type for every tensor of every layer: the single-type kernel; else
    // every layer's gate and up share a type and all types are mixed-stack
    // types: the mixed kernel
    bool one_type = true, mixable = true;
    unsigned used_a = 0, used_b = 0;
    for (int64_t l = 0; l < n_layers; ++l) {
        const moe_layer_desc &Ll = layers[l];
        one_type &= Ll.gate.type == L0.up.type && Ll.up.type == L0.up.type && Ll.down.type == L0.up.type;
        mixable &= Ll.gate.type == Ll.up.type && moe::stack_mix_supported(Ll.up.type) &&
                   moe::stack_mix_supported(Ll.down.type);
        if (mixable) {
            used_a |= 1u << moe::stack_mix_slot(Ll.up.type);
            used_b |= 1u << moe::stack_mix_slot(Ll.down.type);
        }
    }
    const bool mixed = !(one_type && moe::stack_type_supported(L0.up.type, L0.up.type));
    if (mixed && !mixable)
        return fail(MOE_ERR_UNSUPPORTED, "the stack kernel needs one type for gate, up and down, or gate = up and "
                                         "types among Q2_K, Q3_K, Q4_K, Q6_K per layer");
    if (L0.up.ne[0] != L0.H || L0.up.ne[1] != L0.F || L0.down.ne[0] != L0.F || L0.down.ne[1] != L0.H)
        return fail(MOE_ERR_INVALID, "expert tensor shapes do not match H/F");
    const bool shared = L0.shared_type >= 0;
    std::vector<moe::StackLayer> d(static_cast<size_t>(n_layers));
    const LayerWs w = layer_ws(&L0, 1, static_cast<char *>(workspace));
    for (int64_t l = 0; l < n_layers; ++l) {
        const moe_layer_desc &Ll = layers[l];
        const bool same = Ll.H == L0.H && Ll.F == L0.F && Ll.n_experts == L0.n_experts && Ll.k == L0.k &&
                          Ll.glu_op == L0.glu_op && Ll.glu_limit == L0.glu_limit && Ll.norm_w == L0.norm_w &&
                          (Ll.shared_type >= 0) == shared && Ll.up.ne[0] == L0.H && Ll.up.ne[1] == L0.F &&
                          Ll.down.ne[0] == L0.F && Ll.down.ne[1] == L0.H;
        if (!same) return fail(MOE_ERR_INVALID, "layer %lld differs from layer 0 in shape", static_cast<long long>(l));
        const moe_tensor *T[3] = {&Ll.gate, &Ll.up, &Ll.down};
        for (const moe_tensor *t : T)
            if (!t->data || !contiguous(t) || t->ne[2] != Ll.n_experts || !aligned16(t->data) || t->nb[2] % 16 ||
                ptr_kind(t->data) != 2)
                return fail(MOE_ERR_UNSUPPORTED, "stack layers need contiguous, 16-byte aligned expert tensors in device memory");
        if (shared && (!aligned16(Ll.shared_gate) || !aligned16(Ll.shared_up) || !aligned16(Ll.shared_down)))
            return fail(MOE_ERR_UNSUPPORTED, "shared expert data must be 16-byte aligned");
        if (!x[l] || !logits[l] || !out[l]) return fail(MOE_ERR_INVALID, "null x, logits or out of layer %lld", static_cast<long long>(l));
        moe::StackLayer &s = d[static_cast<size_t>(l)];
        s.up = static_cast<const char *>(Ll.up.data);
        s.gate = static_cast<const char *>(Ll.gate.data);
        s.down = static_cast<const char *>(Ll.down.data);
        s.sh_up = shared ? static_cast<const char *>(Ll.shared_up) : nullptr;
        s.sh_gate = shared ? static_cast<const char *>(Ll.shared_gate) : nullptr;
        s.sh_down = shared ? static_cast<const char *>(Ll.shared_down) : nullptr;
        s.x = x[l];
        s.logits = logits[l];
        s.out = out[l];
        s.x_next = x_next ? x_next[l] : nullptr;
        s.ids_out = w.ids;
        s.w_out = w.w;
        s.chained = l > 0 && x_next && x_next[l - 1] == x[l] ? 1 : 0;
        s.ta = mixed ? moe::stack_mix_slot(Ll.up.type) : 0;
        s.tb = mixed ? moe::stack_mix_slot(Ll.down.type) : 0;
    }
    if (mixed) g_stack_mixed[workspace] = {used_a, used_b};
    else g_stack_mixed.erase(workspace);
    const StackWs sw = stack_ws(&L0, n_layers, static_cast<char *>(workspace));
    CK(cudaMemcpyAsync(sw.layers, d.data(), sizeof(moe::StackLayer) * d.size(), cudaMemcpyHostToDevice,
                       reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

int moe_b200_stack_run(const moe_layer_desc *layer0, int64_t n_layers, void *workspace, size_t workspace_bytes,
                       moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!layer0 || n_layers < 1) return fail(MOE_ERR_INVALID, "null argument");
    const size_t need = moe_b200_stack_workspace_size(layer0, n_layers);
    if (!workspace || workspace_bytes < need) return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu)", workspace_bytes, need);
    const auto mix = g_stack_mixed.find(workspace);
    const bool mixed = mix != g_stack_mixed.end();
    if (!mixed && (layer0->gate.type != layer0->up.type ||
                   !moe::stack_type_supported(layer0->up.type, layer0->down.type)))
        return fail(MOE_ERR_UNSUPPORTED, "the stack kernel needs one type for gate, up and down");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const LayerWs w = layer_ws(layer0, 1, static_cast<char *>(workspace));
    // the per-phase shapes and outputs (pointers of layer 0 stand in; the
    // kernel reads every layer's own from its descriptor)
    const float *dummy = reinterpret_cast<const float *>(workspace);
    moe::LayerArgs la;
    int rc = layer_args(layer0, dummy, dummy, const_cast<float *>(dummy), 1, w, st, &la);
    if (rc) return rc;
    moe::StackArgs a{};
    a.gu = la.gu;
    a.dn = la.dn;
    const StackWs sw = stack_ws(layer0, n_layers, static_cast<char *>(workspace));
    a.layers = sw.layers;
    a.n_layers = static_cast<int32_t>(n_layers);
    a.k = static_cast<int32_t>(layer0->k);
    a.n_experts = static_cast<int32_t>(layer0->n_experts);
    a.norm_w = layer0->norm_w;
    a.eb_up = layer0->up.nb[2];
    a.eb_gate = layer0->gate.nb[2];
    a.eb_down = layer0->down.nb[2];
    a.tma = 1;
    a.has_shared = layer0->shared_type >= 0 ? 1 : 0;
    a.h_tag = w.h_tag;
    a.hs_tag = w.hs_tag;
    if (la.dn.stride_channel_dst != layer0->H) return fail(MOE_ERR_INVALID, "unexpected down-row stride");
    a.ysc = layer0->H;
    a.ytag = sw.ytag;
    a.ytag_s = sw.ytag + static_cast<size_t>(layer0->k * layer0->H);
    a.xtag = sw.xtag;
    a.gbar = w.gbar;
    a.err = g.d_err;
    a.timeout_ns = g.timeout_ns_kernel;
    const char *why = "";
    cudaError_t ce = cudaSuccess;
    rc = mixed ? moe::launch_stack_mixed(mix->second.first, mix->second.second, a, st, &why, &ce)
               : moe::launch_stack(layer0->up.type, a, st, &why, &ce);
    if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
    if (rc) return fail(rc, "%s", why);
    return MOE_OK;
}

size_t moe_b200_ep_decode_buffer_bytes(int64_t H, int64_t n_experts, int64_t k, int32_t world) {
    if (H < 1 || n_experts < 1 || k < 1 || world < 1 || world > moe::EP_DECODE_MAX_WORLD) return 0;
    return static_cast<size_t>(moe::ep_decode_layout(static_cast<int>(H), static_cast<int>(n_experts),
                                                     static_cast<int>(k), world).bytes);
}

int moe_b200_ep_layer_decode_p2p(const moe_layer_desc *L, int64_t expert_lo, int64_t n_experts_global,
                                 const void *const *peer_bufs, int32_t world, int32_t rank, const float *x,
                                 const float *logits, float *out, void *workspace, size_t workspace_bytes,
                                 moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !logits || !out || !peer_bufs) return fail(MOE_ERR_INVALID, "null argument");
    if (world < 1 || world > moe::EP_DECODE_MAX_WORLD || rank < 0 || rank >= world)
        return fail(MOE_ERR_INVALID, "world must be 1..%d and 0 <= rank < world", moe::EP_DECODE_MAX_WORLD);
    if (expert_lo < 0 || expert_lo + L->n_experts > n_experts_global || n_experts_global > 65536)
        return fail(MOE_ERR_INVALID, "local experts [%lld, %lld) outside the %lld routed experts",
                    static_cast<long long>(expert_lo), static_cast<long long>(expert_lo + L->n_experts),
                    static_cast<long long>(n_experts_global));
    const int64_t k = L->k, F = L->F, H = L->H;
    if (k < 1 || k > 32 || k > n_experts_global) return fail(MOE_ERR_INVALID, "need 1 <= k <= min(32, n_experts)");
    if (L->up.ne[0] != H || L->up.ne[1] != F || L->down.ne[0] != F || L->down.ne[1] != H)
        return fail(MOE_ERR_INVALID, "expert tensor shapes do not match H/F");
    if (H % 4 || !aligned16(x)) return fail(MOE_ERR_INVALID, "x must be 16-byte aligned with H a multiple of 4");
    for (int32_t r = 0; r < world; ++r)
        if (!peer_bufs[r] || !aligned16(peer_bufs[r])) return fail(MOE_ERR_INVALID, "peer buffer %d null or unaligned", r);
    if (g.layer_fused == 0 || g.layer_fused == 2 || !layer_fusable(L, world))
        return fail(MOE_ERR_UNSUPPORTED, "the fused expert-parallel decode needs the per-expert-group kernel for this layer");
    const LayerWs w = layer_ws(L, world, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes) return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu)", workspace_bytes, w.bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    moe::LayerArgs a;
    int rc = layer_args(L, x, logits, out, world, w, st, &a);
    if (rc) return rc;
    // the shared expert serves this GPU's token only
    a.gu.ncols_dst = a.dn.ncols_dst = 1;
    moe::Layer2Args b = to_layer2(a, w.rowcnt);
    b.n_experts = static_cast<int32_t>(n_experts_global);
    b.ep_on = 1;
    b.ep_timeout_ns = g.timeout_ns_ep;
    b.ep.world = world;
    b.ep.rank = rank;
    b.ep.expert_lo = static_cast<int32_t>(expert_lo);
    b.ep.n_local = static_cast<int32_t>(L->n_experts);
    for (int32_t r = 0; r < world; ++r) b.ep.peer[r] = static_cast<char *>(const_cast<void *>(peer_bufs[r]));
    b.ep.lay = moe::ep_decode_layout(static_cast<int>(H), static_cast<int>(n_experts_global), static_cast<int>(k), world);
    const char *why = "";
    cudaError_t ce = cudaSuccess;
    rc = moe::launch_layer2(L->up.type, L->down.type, b, st, &why, &ce);
    if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
    if (rc) return fail(rc, "%s", why);
    return MOE_OK;
}

int moe_b200_set_wait_limits(int64_t kernel_wait_ns, int64_t exchange_wait_ns) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    constexpr uint64_t kDefault = 2000000000ull;
    g.timeout_ns_kernel = kernel_wait_ns > 0 ? static_cast<uint64_t>(kernel_wait_ns) : kDefault;
    g.timeout_ns_ep = exchange_wait_ns > 0 ? static_cast<uint64_t>(exchange_wait_ns) : kDefault;
    return MOE_OK;
}

int moe_b200_ep_wait(const uint32_t *flag, uint32_t target, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!flag) return fail(MOE_ERR_INVALID, "null flag");
    int rc = ensure_device();
    if (rc) return rc;
    CK(moe::launch_ep_wait(flag, target, g.timeout_ns_ep, g.d_err, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

namespace {

// The received rows' experts: gate and up (one grouping and quantizing
// gather from the f32 rows), down from GLU(gate, up) quantized in the
// gather; every type on the tensor cores. Empty slots (id -1) are skipped.
struct EpRowsWs {
    int32_t *entries, *n_chunks;
    int4 *chunks;
    uint8_t *btiles;
    int64_t max_chunks;
    size_t bytes;
};

EpRowsWs ep_rows_ws(const moe_layer_desc *L, int64_t n_rows, char *base) {
    EpRowsWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
    w.entries = reinterpret_cast<int32_t *>(take(4 * n_rows));
    w.max_chunks = moe::mmq_max_chunks(n_rows, L->n_experts, 32);
    w.chunks = reinterpret_cast<int4 *>(take(16 * static_cast<size_t>(w.max_chunks)));
    w.n_chunks = reinterpret_cast<int32_t *>(take(4));
    const int64_t kmax = L->H > L->F ? L->H : L->F;
    w.btiles = reinterpret_cast<uint8_t *>(take(static_cast<size_t>(w.max_chunks) * (kmax / 256) * moe::MMQ_BT_BYTES));
    w.bytes = off;
    return w;
}

int mmq_call(const moe_tensor *t, const EpRowsWs &w, int64_t n_rows, float *dst, cudaStream_t st) {
    moe::MmqArgs a{};
    a.dense = static_cast<const char *>(t->data);
    a.expert_bytes = t->nb[2];
    a.n_experts = static_cast<int32_t>(t->ne[2]);
    a.K = static_cast<int32_t>(t->ne[0]);
    a.nrows = static_cast<int32_t>(t->ne[1]);
    a.row_bytes = static_cast<uint32_t>(t->nb[1]);
    a.btiles = w.btiles;
    a.n_tok = static_cast<int32_t>(n_rows);
    a.k = 1;
    a.entries = w.entries;
    a.chunks = w.chunks;
    a.n_chunks = w.n_chunks;
    a.dst = dst;
    a.err = g.d_err;
    a.timeout_ns = g.timeout_ns_kernel;
    const char *why = "";
    cudaError_t ce = cudaSuccess;
    const int rc = moe::launch_mmq(t->type, a, st, &why, &ce);
    if (rc == MOE_ERR_CUDA) return fail(rc, "%s: %s", why, cudaGetErrorString(ce));
    if (rc) return fail(rc, "%s", why);
    return MOE_OK;
}

}  // namespace

size_t moe_b200_ep_experts_rows_workspace_size(const moe_layer_desc *L, int64_t n_rows) {
    if (!L || n_rows < 1) return 0;
    return ep_rows_ws(L, n_rows, nullptr).bytes;
}

int moe_b200_ep_experts_rows(const moe_layer_desc *L, const float *x, const int32_t *ids, int64_t n_rows, float *g_out,
                             float *u_out, float *y, void *workspace, size_t workspace_bytes, moe_stream_t stream) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || !x || !ids || !g_out || !u_out || !y || n_rows < 1) return fail(MOE_ERR_INVALID, "null argument");
    for (const moe_tensor *t : {&L->gate, &L->up, &L->down}) {
        if (!moe::mmq_supported(t->type, t->ne[0], t->ne[1]) || moe::mmq_b32(t->type) || !t->data ||
            ptr_kind(t->data) != 2 || !contiguous(t) ||
            !aligned16(t->data) || (t->nb[2] % 16) != 0 || t->ne[2] != L->n_experts)
            return fail(MOE_ERR_UNSUPPORTED, "expert-parallel rows need tensor-core types in device memory");
    }
    const EpRowsWs w = ep_rows_ws(L, n_rows, static_cast<char *>(workspace));
    if (!workspace || workspace_bytes < w.bytes)
        return fail(MOE_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, w.bytes);
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int E = static_cast<int>(L->n_experts), n = static_cast<int>(n_rows);
    int ntc = moe::mmq_chunk_tokens(L->gate.type);
    CK(moe::launch_mmq_group(ids, 1, n, 1, E, ntc, w.entries, w.chunks, w.n_chunks, g.d_err, st, true));
    CK(moe::launch_mmq_gather_rows(x, nullptr, 0, 0.f, static_cast<int>(L->H), w.entries, w.chunks, w.n_chunks, ntc,
                                   w.max_chunks, w.btiles, st));
    rc = mmq_call(&L->gate, w, n_rows, g_out, st);
    if (rc) return rc;
    if (moe::mmq_chunk_tokens(L->up.type) != ntc) {
        ntc = moe::mmq_chunk_tokens(L->up.type);
        CK(moe::launch_mmq_group(ids, 1, n, 1, E, ntc, w.entries, w.chunks, w.n_chunks, g.d_err, st, true));
        CK(moe::launch_mmq_gather_rows(x, nullptr, 0, 0.f, static_cast<int>(L->H), w.entries, w.chunks, w.n_chunks,
                                       ntc, w.max_chunks, w.btiles, st));
    }
    rc = mmq_call(&L->up, w, n_rows, u_out, st);
    if (rc) return rc;
    if (moe::mmq_chunk_tokens(L->down.type) != ntc) {
        ntc = moe::mmq_chunk_tokens(L->down.type);
        CK(moe::launch_mmq_group(ids, 1, n, 1, E, ntc, w.entries, w.chunks, w.n_chunks, g.d_err, st, true));
    }
    CK(moe::launch_mmq_gather_rows(g_out, u_out, L->glu_op, L->glu_limit, static_cast<int>(L->F), w.entries, w.chunks,
                                   w.n_chunks, ntc, w.max_chunks, w.btiles, st));
    return mmq_call(&L->down, w, n_rows, y, st);
}

int moe_b200_layer_fused(const moe_layer_desc *L, int64_t n_tok) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (!L || n_tok < 1 || n_tok > 8 || L->gate.type != L->up.type) return 0;
    return layer_fusable(L, n_tok) ? 1 : 0;
}

int moe_b200_layer_set_fused(int32_t enable) {
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    read_env();
    if (enable < 0 || enable > 2) return fail(MOE_ERR_INVALID, "fused layer mode must be 0, 1 or 2");
    g.layer_fused = enable;
    return MOE_OK;
}

int moe_b200_fill_quantized(int32_t type, void *dst, int64_t n_rows, int64_t n_cols, uint64_t seed, float sigma,
                            moe_stream_t stream) {
    if (!type_supported(type)) return fail(MOE_ERR_UNSUPPORTED, "unsupported type %d", type);
    if (n_cols % blck_size(type)) return fail(MOE_ERR_INVALID, "n_cols not a multiple of the block size");
    CK(moe::launch_fill_quantized(type, dst, n_rows, n_cols, seed, sigma, reinterpret_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

}  // extern "C"
