// moe_noalloc.cu -- a MoE layer decode that allocates nothing.
//
// Some callers cannot call cudaMalloc (or any allocator) at the point where
// they run a layer: a serving engine that reserves all device memory up front
// and owns every byte of it, a plugin whose host framework forbids
// allocations inside its enqueue / compute callback, or code that must not
// trigger the implicit synchronisation an allocation can cause in the middle
// of a decode loop. moe_b200_layer_decode_noalloc serves them: it runs the
// same kernels as moe_b200_layer_decode (routing, fused gate/up GEMV with the
// GLU and the shared expert, down GEMV, weighted combine), but its scratch --
// routing ids and weights, the GLU outputs, the per-pick down outputs, the
// three per-tensor expert pointer tables and a device error word -- lives in
// one file-scope __device__ array of fixed size instead of caller-provided or
// library-allocated memory.
//
// Limits (checked on every call, larger requests are rejected):
//   n_tok <= 8, k <= 8, H <= 4096, F <= 4096, n_experts <= 1024
// which sizes the array at NOALLOC_SCRATCH_BYTES (about 2.3 MB). Every GPU
// that loads the library holds that array until the process exits.
//
// The expert tensors must be in device memory (HBM-resident): the hot-expert
// cache, whose pools and tables are allocated, is not used by this entry
// point, and no bookkeeping (stamps, hit/miss log) is recorded.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (once per device, with that device current); make that
// first call before any stream capture. All calls share the one array and it
// keeps the last call's contents: calls that overlap on the GPU (on different
// streams without ordering between them) race on it.
#include <cstdint>
#include <mutex>

#include "moe_aux.h"
#include "moe_cache_b200.h"
#include "moe_gemv.cuh"

namespace {

constexpr int64_t NA_MAX_TOK = 8, NA_MAX_K = 8, NA_MAX_H = 4096, NA_MAX_F = 4096, NA_MAX_E = 1024;

// scratch layout (byte offsets, each 256-aligned)
constexpr size_t na_align(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
constexpr size_t NA_IDS = 0;
constexpr size_t NA_W = NA_IDS + na_align(sizeof(int32_t) * NA_MAX_TOK * NA_MAX_K);
constexpr size_t NA_H = NA_W + na_align(sizeof(float) * NA_MAX_TOK * NA_MAX_K);
constexpr size_t NA_HS = NA_H + na_align(sizeof(float) * NA_MAX_TOK * NA_MAX_K * NA_MAX_F);
constexpr size_t NA_Y = NA_HS + na_align(sizeof(float) * NA_MAX_TOK * NA_MAX_F);
constexpr size_t NA_YS = NA_Y + na_align(sizeof(float) * NA_MAX_TOK * NA_MAX_K * NA_MAX_H);
constexpr size_t NA_TBL = NA_YS + na_align(sizeof(float) * NA_MAX_TOK * NA_MAX_H);
constexpr size_t NA_ERR = NA_TBL + na_align(sizeof(char *) * 3 * NA_MAX_E);
constexpr size_t NOALLOC_SCRATCH_BYTES = NA_ERR + 256;

}  // namespace

// The scratch. In host code this name is only a host-side stand-in for the
// symbol, not a device address: the kernels get the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_na_mu;
unsigned char *g_na_ptr[64] = {nullptr};   // device address of the scratch, per device

// Fills the three expert tables (expert e of a contiguous tensor starts at
// base + e * expert_bytes) and clears the error word.
__global__ void noalloc_tables_kernel(char **tbl, const char *gate, const char *up, const char *down, uint64_t eb_gate,
                                      uint64_t eb_up, uint64_t eb_down, int n_experts, int *err) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e == 0) *err = 0;
    if (e >= n_experts) return;
    tbl[e] = const_cast<char *>(gate) + static_cast<uint64_t>(e) * eb_gate;
    tbl[NA_MAX_E + e] = const_cast<char *>(up) + static_cast<uint64_t>(e) * eb_up;
    tbl[2 * NA_MAX_E + e] = const_cast<char *>(down) + static_cast<uint64_t>(e) * eb_down;
}

int na_type_size(int t) {
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

bool na_on_device(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) { cudaGetLastError(); return false; }
    int dev = 0;
    cudaGetDevice(&dev);
    return at.type == cudaMemoryTypeDevice && at.device == dev;
}

bool na_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool na_contiguous(const moe_tensor &t) {
    const uint64_t ts = static_cast<uint64_t>(na_type_size(t.type));
    const int64_t bs = (t.type >= MOE_TYPE_Q2_K && t.type <= MOE_TYPE_Q6_K) ? 256 : 32;
    if (!ts || t.ne[0] % bs) return false;
    return t.nb[0] == ts && t.nb[1] == ts * static_cast<uint64_t>(t.ne[0] / bs) &&
           t.nb[2] == t.nb[1] * static_cast<uint64_t>(t.ne[1]);
}

}  // namespace

extern "C" int moe_b200_layer_decode_noalloc(const moe_layer_desc *L, const float *x, const float *logits, float *out,
                                             int64_t n_tok, moe_stream_t stream) {
    if (!L || !x || !logits || !out) return MOE_ERR_INVALID;
    if (n_tok < 1 || n_tok > NA_MAX_TOK || L->k < 1 || L->k > NA_MAX_K || L->H < 1 || L->H > NA_MAX_H || L->F < 1 ||
        L->F > NA_MAX_F || L->n_experts < 1 || L->n_experts > NA_MAX_E)
        return MOE_ERR_UNSUPPORTED;   // beyond the fixed scratch: n_tok<=8, k<=8, H<=4096, F<=4096, n_experts<=1024
    const int64_t H = L->H, F = L->F, k = L->k;
    const moe_tensor *T[3] = {&L->gate, &L->up, &L->down};
    for (const moe_tensor *t : T) {
        if (!t->data || !na_contiguous(*t) || t->ne[2] != L->n_experts || !na_aligned16(t->data) || !na_on_device(t->data))
            return MOE_ERR_UNSUPPORTED;   // expert tensors: contiguous, 16-byte aligned, in device memory
    }
    if (L->gate.type != L->up.type || L->up.ne[0] != H || L->up.ne[1] != F || L->gate.ne[0] != H || L->gate.ne[1] != F ||
        L->down.ne[0] != F || L->down.ne[1] != H)
        return MOE_ERR_INVALID;
    const bool shared = L->shared_type >= 0;
    if (shared && (!L->shared_gate || !L->shared_up || !L->shared_down || !na_aligned16(L->shared_gate) ||
                   !na_aligned16(L->shared_up) || !na_aligned16(L->shared_down)))
        return MOE_ERR_INVALID;

    std::lock_guard<std::mutex> lock(g_na_mu);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_CUDA;
    if (!g_na_ptr[dev]) {
        // set-up, once per device, with that device current
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return MOE_ERR_CUDA;
        }
        g_na_ptr[dev] = static_cast<unsigned char *>(p);
    }
    unsigned char *base = g_na_ptr[dev];
    int32_t *ids = reinterpret_cast<int32_t *>(base + NA_IDS);
    float *w = reinterpret_cast<float *>(base + NA_W);
    float *h = reinterpret_cast<float *>(base + NA_H);
    float *hs = reinterpret_cast<float *>(base + NA_HS);
    float *y = reinterpret_cast<float *>(base + NA_Y);
    float *ys = reinterpret_cast<float *>(base + NA_YS);
    char **tbl = reinterpret_cast<char **>(base + NA_TBL);
    int *err = reinterpret_cast<int *>(base + NA_ERR);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    const int E = static_cast<int>(L->n_experts);
    noalloc_tables_kernel<<<(E + 255) / 256, 256, 0, st>>>(tbl, static_cast<const char *>(L->gate.data),
                                                           static_cast<const char *>(L->up.data),
                                                           static_cast<const char *>(L->down.data), L->gate.nb[2],
                                                           L->up.nb[2], L->down.nb[2], E, err);
    if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
    if (moe::launch_topk_softmax(logits, n_tok, L->n_experts, k, L->norm_w, ids, w, st) != cudaSuccess)
        return MOE_ERR_CUDA;

    const char *why = "";
    cudaError_t ce = cudaSuccess;
    // fused gate/up GEMV with the GLU and the shared expert
    moe::GemvArgs a{};
    a.tbl = tbl + NA_MAX_E;
    a.tbl_gate = tbl;
    a.use_gate = 1;
    a.has_fusion = 1;
    a.glu_op = L->glu_op;
    a.glu_limit = L->glu_limit;
    a.tma_main = (L->up.nb[2] % 16) == 0;
    a.tma_gate = (L->gate.nb[2] % 16) == 0;
    if (shared) {
        a.shared_up = static_cast<const char *>(L->shared_up);
        a.shared_gate = static_cast<const char *>(L->shared_gate);
        a.shared_dst = hs;
        a.shared_stride_col_dst = F;
        a.tma_shared = (L->up.nb[2] % 16) == 0 && na_on_device(L->shared_up) && na_on_device(L->shared_gate);
    }
    a.y = x;
    a.stride_col_y = H;
    a.stride_channel_y = 0;
    a.nchannels_y = 1;
    a.ids = ids;
    a.ids_stride = k;
    a.ncols_dst = static_cast<int32_t>(n_tok);
    a.nchannels_dst = static_cast<int32_t>(k);
    a.n_experts = E;
    a.dst = h;
    a.stride_col_dst = k * F;
    a.stride_channel_dst = F;
    a.K = static_cast<int32_t>(H);
    a.nrows = static_cast<int32_t>(F);
    a.row_bytes = static_cast<uint32_t>(L->up.nb[1]);
    a.err = err;
    int rc = moe::launch_gemv(L->up.type, moe::ACT_CPU, a, st, &why, &ce);
    if (rc) return rc;

    // down GEMV (the shared expert's down projection reads hs)
    moe::GemvArgs d{};
    d.tbl = tbl + 2 * NA_MAX_E;
    d.tma_main = (L->down.nb[2] % 16) == 0;
    if (shared) {
        d.shared_up = static_cast<const char *>(L->shared_down);
        d.shared_dst = ys;
        d.shared_stride_col_dst = H;
        d.shared_y = hs;
        d.shared_y_stride_col = F;
        d.tma_shared = (L->down.nb[2] % 16) == 0 && na_on_device(L->shared_down);
    }
    d.y = h;
    d.stride_col_y = k * F;
    d.stride_channel_y = F;
    d.nchannels_y = static_cast<int32_t>(k);
    d.ids = ids;
    d.ids_stride = k;
    d.ncols_dst = static_cast<int32_t>(n_tok);
    d.nchannels_dst = static_cast<int32_t>(k);
    d.n_experts = E;
    d.dst = y;
    d.stride_col_dst = k * H;
    d.stride_channel_dst = H;
    d.K = static_cast<int32_t>(F);
    d.nrows = static_cast<int32_t>(H);
    d.row_bytes = static_cast<uint32_t>(L->down.nb[1]);
    d.err = err;
    rc = moe::launch_gemv(L->down.type, moe::ACT_CPU, d, st, &why, &ce);
    if (rc) return rc;
    if (moe::launch_combine(y, w, shared ? ys : nullptr, out, n_tok, H, k, st) != cudaSuccess) return MOE_ERR_CUDA;
    return MOE_OK;
}

// No counterpart in the reference: read the no-alloc path's device error word
// (0 = none) after synchronising `stream`. It is not cleared here: the next
// no-alloc call clears it (noalloc_tables_kernel).
extern "C" int moe_b200_noalloc_device_error(moe_stream_t stream, int32_t *code) {
    if (code) *code = 0;
    std::lock_guard<std::mutex> lock(g_na_mu);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_CUDA;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (!g_na_ptr[dev]) return cudaStreamSynchronize(st) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
    // read on the caller's stream (after its work), not on the legacy stream,
    // which would wait for every other stream of the device too
    int v = 0;
    if (cudaMemcpyAsync(&v, g_na_ptr[dev] + NA_ERR, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return MOE_ERR_CUDA;
    if (code) *code = v;
    return MOE_OK;
}
