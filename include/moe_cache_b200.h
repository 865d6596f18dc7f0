/*
 * moe_cache_b200.h -- C ABI of the B200 (sm_100a) MoE expert hot path.
 *
 * The entry points named ggml_cuda_moe_cache_* are the reference's boundary
 * (kernels/moe-cache.cuh:15-40 of Zapdev-labs/a6000-custom-kernels) restated as
 * a C ABI: plain pointers and sizes instead of ggml_tensor / C++ references,
 * and an int status instead of aborting. Entry points prefixed moe_b200_ are
 * additions with no reference counterpart; each says so.
 *
 * Status: 0 = MOE_OK, negative = error (moe_b200_last_error() describes it).
 * Threading: all entry points are serialised by one library mutex, as the
 * reference serialises its registry and step (moe-cache.cu:321,526,674).
 * Streams: all work is enqueued on the caller's stream, as in the reference.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *moe_stream_t;   /* same type as cudaStream_t */

#define MOE_OK               0
#define MOE_ERR_INVALID     -1   /* bad argument or shape */
#define MOE_ERR_UNSUPPORTED -2   /* type / layout the path does not handle */
#define MOE_ERR_CUDA        -3   /* a CUDA runtime call failed */
#define MOE_ERR_OOM         -4   /* allocation failed */
#define MOE_ERR_DEVICE      -5   /* a kernel reported a device-side check failure */
#define MOE_ERR_STATE       -6   /* called in the wrong state (e.g. wrong device) */

/* ggml_type numbering (ggml.h) for the formats of the path */
enum {
    MOE_TYPE_F32 = 0, MOE_TYPE_Q4_0 = 2, MOE_TYPE_Q5_0 = 6, MOE_TYPE_Q8_0 = 8, MOE_TYPE_Q8_1 = 9,
    MOE_TYPE_Q2_K = 10, MOE_TYPE_Q3_K = 11, MOE_TYPE_Q4_K = 12, MOE_TYPE_Q5_K = 13,
    MOE_TYPE_Q6_K = 14, MOE_TYPE_Q8_K = 15,
};

/* GLU ops of the fused gate/up epilogue (moe-cache.cu:264-280). The shim maps
 * ggml_glu_op by name: SWIGLU, GEGLU, SWIGLU_OAI, SWIGLU_CLAMP; every other op
 * maps to MOE_GLU_PRODUCT, which is the reference's default branch. */
enum { MOE_GLU_SWIGLU = 0, MOE_GLU_GEGLU = 1, MOE_GLU_SWIGLU_OAI = 2, MOE_GLU_SWIGLU_CLAMP = 3,
       MOE_GLU_PRODUCT = 4 };

#define MOE_TENSOR_VIEW      1   /* ggml_tensor::view_src != NULL */
#define MOE_TENSOR_NO_BUFFER 2   /* ggml_tensor::buffer == NULL   */

/* The fields of a ggml_tensor that the path reads. */
typedef struct {
    const void *data;
    int32_t     type;      /* MOE_TYPE_* */
    int32_t     flags;     /* MOE_TENSOR_* */
    int64_t     ne[4];
    uint64_t    nb[4];
    const char *name;      /* NUL-terminated; matched against seed-file lines */
} moe_tensor;

/* Mirror of upstream ggml_cuda_mm_fusion_args_host: the gate tensor, which
 * gets its own table when it is itself cached (moe-cache.cu:840-844). */
typedef struct {
    const moe_tensor *gate;   /* may be NULL */
} moe_fusion_host;

/* Mirror of upstream ggml_cuda_mm_fusion_args_device (fields read at
 * moe-cache.cu:103-129,797-798). All pointers are device pointers. */
typedef struct {
    const void  *gate;        /* gate weights, used when the gate has no table  */
    const float *x_bias;      /* [n_experts][rows], added to the up/main result */
    const float *gate_bias;   /* [n_experts][rows], added to the gate result    */
    const float *x_scale;     /* NVFP4-only upstream: accepted and ignored      */
    const float *gate_scale;  /* NVFP4-only upstream: accepted and ignored      */
    int32_t      glu_op;      /* MOE_GLU_*                                      */
    float        glu_limit;
    const void  *shared_up;   /* shared expert ([rows][row bytes], same type)   */
    const void  *shared_gate;
    float       *shared_dst;
    int64_t      shared_stride_col_dst;
} moe_fusion_device;

/* Replaces: bool ggml_cuda_moe_cache_enabled()  (moe-cache.cuh:15,
 * moe-cache.cu:345-363). Reads GGML_CUDA_MOE_CACHE, _SLOTS, _BUDGET_GB,
 * _SEED, _DEBUG and _DEVICE once. Returns 1 when enabled, 0 otherwise. */
int ggml_cuda_moe_cache_enabled(void);

/* Replaces: bool ggml_cuda_moe_cache_wants(const ggml_tensor*)  (moe-cache.cuh:18,
 * moe-cache.cu:442-469). 1 when src0 should take this path: enabled, supported
 * type, ne[2] >= 2, ne[3] == 1, not a view, contiguous, and either pinned host
 * memory (tiered cache, as in the reference) or device memory (HBM-resident
 * experts, new on B200; off with GGML_CUDA_MOE_CACHE_DEVICE=0). */
int ggml_cuda_moe_cache_wants(const moe_tensor *src0);

/* Replaces: void ggml_cuda_moe_cache_mul_mat_vec_q(ctx, src0, ids, dst, fusion,
 * fusion_dev, src1_q8_1, ids_d, dst_d, ne00..ne03, ncols_dst, s01..s03,
 * nchannels_y, nchannels_dst, stride_col_y, stride_col_dst, stride_channel_y,
 * stride_channel_dst, ids_stride, stream)  (moe-cache.cuh:21-30,
 * moe-cache.cu:821-868). The unused ctx/ids/dst tensor arguments are dropped.
 *
 * dst_d[ch*stride_channel_dst + tok*stride_col_dst + row] =
 *     dot(expert ids_d[ch + tok*ids_stride] row `row`, src1[(ch % nchannels_y), tok])
 * for ch < nchannels_dst, tok < ncols_dst, row < ne01, with the fused gate /
 * GLU / bias / shared-expert epilogue when fusion_dev enables it.
 *
 * src1_type selects the activation semantics:
 *   MOE_TYPE_Q8_1: src1 is Q8_1 blocks (36 B) as produced by llama.cpp's CUDA
 *                  quantize_q8_1 (the reference's input); strides in blocks.
 *   MOE_TYPE_F32:  src1 is f32; the kernel quantizes it exactly as llama.cpp's
 *                  CPU path does (Q8_K for K-quants, Q8_0 for Q4_0/Q5_0/Q8_0);
 *                  strides in floats.
 * ncols_dst <= 8 (the MMVQ batch limit the reference runs at). */
int ggml_cuda_moe_cache_mul_mat_vec_q(
        const moe_tensor *src0, const moe_fusion_host *fusion, const moe_fusion_device *fusion_dev,
        const void *src1, int32_t src1_type, const int32_t *ids_d, float *dst_d,
        int64_t ne00, int64_t ne01, int64_t ne02, int64_t ne03,
        int64_t ncols_dst, int64_t s01, int64_t s02, int64_t s03,
        int64_t nchannels_y, int64_t nchannels_dst,
        int64_t stride_col_y, int64_t stride_col_dst,
        int64_t stride_channel_y, int64_t stride_channel_dst,
        int64_t ids_stride, moe_stream_t stream);

/* Replaces: void ggml_cuda_moe_cache_step(cudaStream_t)  (moe-cache.cuh:33,
 * moe-cache.cu:669-775). Between graphs, never during stream capture. Returns
 * at once (no device sync) when no registered tensor is host-tiered. */
int ggml_cuda_moe_cache_step(moe_stream_t stream);

/* Replaces: bool ggml_cuda_moe_cache_active()  (moe-cache.cuh:36, :365-368). */
int ggml_cuda_moe_cache_active(void);

/* Replaces: bool ggml_cuda_moe_cache_pin_host(const ggml_tensor*)
 * (moe-cache.cuh:39, :372-405). 1 when t->data is GPU-readable host memory
 * after the call (registers a plain host range with cudaHostRegister). */
int ggml_cuda_moe_cache_pin_host(const moe_tensor *t);

/* ---- additions (no counterpart in the reference) ------------------------ */

typedef struct {
    int32_t     enabled;        /* GGML_CUDA_MOE_CACHE            */
    int32_t     slots;          /* GGML_CUDA_MOE_CACHE_SLOTS      (default 320) */
    double      budget_gb;      /* GGML_CUDA_MOE_CACHE_BUDGET_GB  (default 30, <=0 keeps default) */
    const char *seed_path;      /* GGML_CUDA_MOE_CACHE_SEED       (NULL: none)  */
    int32_t     claim_device;   /* GGML_CUDA_MOE_CACHE_DEVICE     (default 1)   */
    int32_t     debug;          /* GGML_CUDA_MOE_CACHE_DEBUG                    */
} moe_cache_config;

/* No counterpart in the reference: set the configuration programmatically
 * instead of from the environment (forgets earlier registrations first). */
int moe_b200_configure(const moe_cache_config *cfg);

/* No counterpart in the reference (its state lives for the process): free all
 * pools, tables and stamps and forget every registration. The next call
 * re-reads the environment unless moe_b200_configure is called. */
int moe_b200_reset(void);

typedef struct {
    uint64_t steps, hits, misses, promotions, evictions, resident, registered, log_overflow;
    uint64_t pool_bytes;
} moe_cache_stats;

/* No counterpart in the reference (it prints every 64 steps): totals. */
int moe_b200_stats(moe_cache_stats *out);

/* No counterpart in the reference: read the DEVICE pointer table of the
 * registered tensor whose data pointer is `data` back to the host and decode
 * it: slot_of[e] = pool slot, -1 = host-tagged (cold), -2 = direct device
 * pointer (HBM-resident tensor). Synchronises the device. */
int moe_b200_table(const void *data, int32_t *slot_of, int32_t n_experts, int32_t *n_slots, int32_t *tensor_id);

/* No counterpart in the reference: synchronise `stream`, then read and clear
 * the kernels' device-side error word (0 = none). */
int moe_b200_device_error(moe_stream_t stream, int32_t *code);

/* No counterpart in the reference: limits of the bounded device-side waits,
 * in nanoseconds; a value <= 0 restores the default of 2 s. kernel_wait_ns
 * bounds the waits inside the GEMV, layer and prefill kernels (a weight tile
 * landing, a ring stage coming free, another CTA's results); exchange_wait_ns
 * bounds moe_b200_ep_wait and the layer kernels' waits for other GPUs. A
 * wait that runs out sets the device error word (moe_b200_device_error:
 * DERR_TIMEOUT_* codes) and its kernel returns once the copies it has in
 * flight have landed (that last wait is never shorter than 200 ms); the
 * context stays usable. Applies to launches issued after the call. */
int moe_b200_set_wait_limits(int64_t kernel_wait_ns, int64_t exchange_wait_ns);

/* Device error codes read by moe_b200_device_error. */
#define MOE_DERR_BAD_ID          1   /* an expert id outside [0, n_experts) */
#define MOE_DERR_TOO_MANY_KEYS   2
#define MOE_DERR_TIMEOUT_FULL    3   /* a wait for data (a weight tile, another GPU's arrivals) ran out */
#define MOE_DERR_TIMEOUT_EMPTY   4   /* a wait for a free ring stage ran out */
#define MOE_DERR_TOO_MANY_SEGMENTS 5
#define MOE_DERR_DRAIN           6   /* copies in flight did not land before exit */
#define MOE_DERR_GRID_BARRIER    7
#define MOE_DERR_TIMEOUT_TAG     8   /* a wait for another CTA's results ran out */
#define MOE_DERR_EP_OVERFLOW     9   /* an expert-parallel receive region was full */

/* No counterpart in the reference: message of the last failed call. */
const char *moe_b200_last_error(void);

/* No counterpart in the reference (upstream quantize_q8_1 / CPU quantizers):
 * quantize n_rows rows of n_cols f32 into act_type blocks (MOE_TYPE_Q8_0,
 * MOE_TYPE_Q8_1 or MOE_TYPE_Q8_K), bit-exact with llama.cpp's quantizers. */
int moe_b200_quantize_act(int32_t act_type, const float *x, void *y, int64_t n_rows, int64_t n_cols,
                          moe_stream_t stream);

/* No counterpart in the reference (upstream graph ops): top-k over logits
 * (descending, ties to the lower expert id) and softmax gating weights. */
int moe_b200_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts, int64_t k, int32_t norm_w,
                          int32_t *ids, float *weights, moe_stream_t stream);

/* One MoE FFN layer (gate/up/down expert tensors + optional shared expert). */
typedef struct {
    moe_tensor  gate, up, down;        /* expert tensors: [E][F][H], [E][F][H], [E][H][F] */
    int32_t     shared_type;           /* -1: no shared expert; otherwise the shared gate, up
                                          and down have gate.type, up.type and down.type */
    const void *shared_gate, *shared_up, *shared_down;
    int64_t     H, F, n_experts, k;
    int32_t     glu_op;
    float       glu_limit;
    int32_t     norm_w;
} moe_layer_desc;

/* No counterpart in the reference: bytes of caller-owned device workspace
 * moe_b200_layer_decode needs for n_tok tokens. Zero-fill the workspace once
 * before its first use (cudaMemset): its first 256 bytes hold the fused
 * kernels' launch epoch, which tags the data their CTAs exchange, then come
 * uint32[8][H / 64 rounded up]: rows of output arrived per (token, block of
 * 64 rows), which the per-expert-group kernel leaves at zero after every
 * launch (a workspace shared by several layers must serve layers of one H).
 * Then (each part 256-byte aligned): ids int32[n][k], weights f32[n][k],
 * h f32[n][k][F], hs f32[n][F], y f32[n][k][H], ys f32[n][H], then the
 * fused kernel's tagged copies of h and hs, then the gate outputs when gate
 * and up differ in type (f32[n][k][F], f32[n][F]). After a launch that
 * reported a device error, zero the workspace again. */
size_t moe_b200_layer_workspace_size(const moe_layer_desc *layer, int64_t n_tok);

/* No counterpart in the reference (the upstream graph around two
 * MUL_MAT_ID calls): one MoE layer for n_tok <= 8 decode tokens, f32 in/out on
 * device: route, fused gate/up GEMV + GLU, down GEMV, weighted combine plus the
 * shared expert; gate and up of different types run as two GEMVs and a GLU
 * pass (as llama.cpp does). Activations use llama.cpp CPU semantics (see
 * src1_type F32).
 * Allocates nothing: `workspace` is caller-owned device memory (zero-filled
 * before first use). Where moe_b200_layer_fused says so, the whole layer is
 * ONE cooperative kernel launch (one CTA per SM; see moe_b200_layer_set_fused
 * for its two forms); otherwise four launches (routing, gate/up, down,
 * combine). All give the same bits. Concurrent calls must not share a
 * workspace. */
int moe_b200_layer_decode(const moe_layer_desc *layer, const float *x, const float *logits, float *out,
                          int64_t n_tok, void *workspace, size_t workspace_bytes, moe_stream_t stream);

/* No counterpart in the reference: the expert-parallel share of one MoE
 * layer decode. `layer` describes THIS GPU's experts: its gate/up/down tensors
 * hold n_experts = E_local experts, global experts [expert_lo, expert_lo +
 * E_local) of the n_experts_global the router picks from. Every GPU routes the
 * same tokens over all experts (same logits, same picks and weights), runs
 * the GEMVs on the picks it holds, and writes its share of the weighted sum to
 * `out` (its picks in pick order, plus the shared expert when with_shared);
 * the caller sums the shares over GPUs (e.g. an NCCL all-reduce). Workspace
 * as moe_b200_layer_decode. Gate and up must share a type. */
int moe_b200_ep_layer_decode(const moe_layer_desc *layer, int64_t expert_lo, int64_t n_experts_global,
                             int32_t with_shared, const float *x, const float *logits, float *out, int64_t n_tok,
                             void *workspace, size_t workspace_bytes, moe_stream_t stream);

/* Prefill MUL_MAT_ID. No counterpart in the reference, which leaves batches
 * above its GEMV limit to llama.cpp's MMQ (patches/apply_patches.py:81-87):
 * dst[(t * k + p) * rows + r] = row r of expert ids[t * ids_stride + p] . x[t]
 * for n_tok tokens (x f32 [n_tok][ne00], contiguous, 16-byte aligned), with
 * llama.cpp CPU semantics (Q8_K activations for K-quants, Q8_0 for Q4_0,
 * Q5_0 and Q8_0). Experts of all 8 types with rows a multiple of 128 (ne00 <=
 * 4096 for K-quants, <= 8192 otherwise) run as a grouped int8 GEMM on the
 * tensor cores with exact integer block dots: Q2_K, Q4_0, Q5_0 and Q8_0 results
 * equal the CPU path bit for bit, Q3_K..Q6_K differ only in the order of float
 * sums. For a host-tiered tensor the picks of experts in its device pool run
 * there (the pool as the expert array), the other picks through the decode
 * GEMV reading pinned host memory in place; other shapes run the GEMV over
 * chunks of 8 tokens. *used_tensor_cores (optional) reports whether the
 * tensor cores ran. Workspace: moe_b200_prefill_workspace_size bytes of device
 * memory, no initialisation needed. */
size_t moe_b200_prefill_workspace_size(const moe_tensor *src0, int64_t n_tok, int64_t k);
int moe_b200_prefill_mul_mat_id(const moe_tensor *src0, const float *x, int64_t n_tok, const int32_t *ids,
                                int64_t k, int64_t ids_stride, float *dst, void *workspace, size_t workspace_bytes,
                                int32_t *used_tensor_cores, moe_stream_t stream);

/* No counterpart in the reference (the upstream graph around two
 * MUL_MAT_ID calls, for a prompt): one MoE layer for any n_tok, f32 in/out on
 * device: route, gate and up per pick (tensor-core prefill MUL_MAT_ID), GLU,
 * down per pick, the shared expert as a one-expert MUL_MAT_ID of every
 * token, weighted combine. Workspace: moe_b200_layer_prefill_workspace_size
 * bytes of device memory (no initialisation needed); allocates nothing. */
size_t moe_b200_layer_prefill_workspace_size(const moe_layer_desc *layer, int64_t n_tok);
int moe_b200_layer_prefill(const moe_layer_desc *layer, const float *x, const float *logits, float *out,
                           int64_t n_tok, void *workspace, size_t workspace_bytes, moe_stream_t stream);

/* No counterpart in the reference: the expert part of a layer prefill,
 * y[t][p] = down_e(GLU(gate_e . x, up_e . x)) with e = ids[t * k + p] for
 * n_tok tokens of k picks (x f32 [n_tok][H], or [n_tok][k][H] with
 * x_per_pick; y f32 [n_tok][k][H]); no routing, shared expert or combine. An
 * expert-parallel GPU runs it on the rows other GPUs sent it (k = 1, ids
 * local to its experts). Workspace: moe_b200_experts_prefill_workspace_size. */
size_t moe_b200_experts_prefill_workspace_size(const moe_layer_desc *layer, int64_t n_tok, int64_t k);
int moe_b200_experts_prefill(const moe_layer_desc *layer, const float *x, int32_t x_per_pick, const int32_t *ids,
                             int64_t n_tok, int64_t k, float *y, void *workspace, size_t workspace_bytes,
                             moe_stream_t stream);

/* No counterpart in the reference: the shared expert of every token,
 * ys f32 [n_tok][H]; workspace as moe_b200_layer_prefill. */
int moe_b200_shared_prefill(const moe_layer_desc *layer, const float *x, int64_t n_tok, float *ys, void *workspace,
                            size_t workspace_bytes, moe_stream_t stream);

/* No counterpart in the reference (upstream graph ops): out[t] = sum over p
 * in order of weights[t][p] * y[t][p] (+ ys[t] when ys is not null). */
int moe_b200_combine(const float *y, const float *weights, const float *ys, float *out, int64_t n_tok, int64_t H,
                     int64_t k, moe_stream_t stream);

/* No counterpart in the reference: expert-parallel prefill exchange over
 * NVLink peer memory (no host round trip per layer). Every GPU allocates its
 * exchange buffers with moe_b200_ipc_alloc (zero-filled; cudaMalloc'd so a
 * CUDA IPC handle covers exactly the buffer), shares handles
 * (moe_b200_ipc_handle, MOE_IPC_HANDLE_BYTES each) and opens the others'
 * (moe_b200_ipc_open). Per GPU: x f32 [W * cap][H] received rows (region s:
 * rows from GPU s; cap = entries per GPU, n_tok * k), ids int32 [W * cap]
 * (local expert, -1 = empty), src int32 [W * cap] (entry t * k + p at the
 * source), y_ret f32 [cap][H] (this GPU's entries' outputs), flags uint32[2]
 * (dispatch and return arrivals, counting up). peer_ptrs is a host array
 * [5][W] of those five pointers for every GPU as seen from the caller.
 * moe_b200_ep_dispatch writes this GPU's entries into their owners' regions
 * and counts one arrival at every GPU; moe_b200_ep_wait (a bounded device
 * wait; timeout -> device error word) holds the stream until a counter
 * reaches target (W per layer call); moe_b200_ep_experts_rows runs an
 * owner's experts on its received rows (gate, up, GLU, down on the tensor
 * cores; empty slots skipped); moe_b200_ep_return writes the outputs back
 * into the sources' y_ret and counts one return arrival at every GPU.
 * scratch: 16 zeroed uint32 of device memory per GPU. */
#define MOE_IPC_HANDLE_BYTES 64
int moe_b200_ipc_alloc(size_t bytes, void **ptr);
int moe_b200_ipc_free(void *ptr);
int moe_b200_ipc_handle(const void *ptr, void *handle);
int moe_b200_ipc_open(const void *handle, void **ptr);
int moe_b200_ipc_close(void *ptr);
int moe_b200_ep_dispatch(const void *const *peer_ptrs, int32_t world, int32_t rank, int64_t cap, const int32_t *ids,
                         int64_t n_entries, int64_t k, int64_t n_experts, const float *x, int64_t H, void *scratch,
                         moe_stream_t stream);
int moe_b200_ep_wait(const uint32_t *flag, uint32_t target, moe_stream_t stream);
size_t moe_b200_ep_experts_rows_workspace_size(const moe_layer_desc *layer, int64_t n_rows);
int moe_b200_ep_experts_rows(const moe_layer_desc *layer, const float *x, const int32_t *ids, int64_t n_rows,
                             float *gate_out, float *up_out, float *y, void *workspace, size_t workspace_bytes,
                             moe_stream_t stream);
int moe_b200_ep_return(const void *const *peer_ptrs, int32_t world, int64_t cap, const int32_t *ids,
                       const int32_t *src, const float *y, int64_t H, void *scratch, moe_stream_t stream);

/* No counterpart in the reference: n_layers batch-1 layers in ONE persistent
 * launch (moe_stack_kernel). Layer l reads its token from x[l] and its router
 * logits from logits[l], writes its output to out[l] and, when x_next (may be
 * NULL) has a non-null entry, x_next[l] = x[l] + out[l] -- so x[l + 1] may be
 * x_next[l] and the layers form a residual chain: every layer starts only
 * after the previous layer's output is complete. Each layer computes what
 * moe_b200_layer_decode computes for one token (same bits). The router logits
 * of every layer are inputs, so each CTA routes layer l + 1 and streams its
 * weights while layer l computes; consecutive layers hand over through tagged
 * words in the workspace (no atomics, no grid barrier). One launch also keeps
 * the code warm in the instruction caches and has no launch gaps. Up to 32
 * picks per layer.
 * Requirements: either gate, up and down of every layer of one type (Q2_K..
 * Q6_K, Q4_0, Q5_0, Q8_0, Q5_K), or per layer gate = up and the gate/up and
 * down types each among Q2_K, Q3_K, Q4_K, Q6_K (a mixed stack: one kernel
 * that picks each layer's types at run time); every layer with layer 0's
 * shapes, GLU and shared-expert presence (the shared expert takes its
 * layer's types), expert tensors contiguous and 16-byte aligned in device
 * memory (no host-tiered tensors, no cache bookkeeping). x, logits, out,
 * x_next are host arrays of n_layers device pointers.
 * moe_b200_stack_prepare writes the layer list into the workspace (an
 * asynchronous copy on `stream` from host memory: not during stream
 * capture) and records, for a mixed stack, the types in use under the
 * workspace's address; moe_b200_stack_run launches (capturable) and may be
 * repeated for the same list. Workspace:
 * moe_b200_stack_workspace_size(layer 0, n_layers) bytes, zero-filled once
 * (its start is a layer-decode workspace for one token). */
size_t moe_b200_stack_workspace_size(const moe_layer_desc *layer0, int64_t n_layers);
int moe_b200_stack_prepare(const moe_layer_desc *layers, int64_t n_layers, const float *const *x,
                           const float *const *logits, float *const *out, float *const *x_next, void *workspace,
                           size_t workspace_bytes, moe_stream_t stream);
int moe_b200_stack_run(const moe_layer_desc *layer0, int64_t n_layers, void *workspace, size_t workspace_bytes,
                       moe_stream_t stream);

/* No counterpart in the reference (the reference runs on one GPU): one MoE
 * layer decode with the experts sharded over `world` GPUs of one node and the
 * exchange fused into the per-expert-group layer kernel, one launch per GPU
 * per layer, no host round trip. GPU r holds global experts [expert_lo,
 * expert_lo + layer->n_experts) of n_experts_global (its gate/up/down
 * tensors hold just those) and the shared expert, and brings ONE token: x
 * f32 [H] and its router logits f32 [n_experts_global]; `out` f32 [H]
 * receives that token's layer output. Each GPU allocates one exchange buffer
 * of moe_b200_ep_decode_buffer_bytes with moe_b200_ipc_alloc (zero-filled),
 * shares its handle and opens the others'; peer_bufs[r] is GPU r's buffer as
 * seen from the caller. In the kernel each GPU writes its token into every
 * GPU's gather slot (peer stores over NVLink, one slot per source, double
 * buffered by call parity) and waits for all of them; routes every token;
 * runs its own experts for every token that picked them (per-expert CTA
 * groups) and the shared expert for its own token; writes each routed down
 * row into the token's GPU; and sums its own token's rows in pick order once
 * they have all arrived. Every value crosses as one 64-bit word (f32 bits |
 * call tag << 32), so a reader that sees the tag sees the value: no fences,
 * no counters. Waits for other GPUs are
 * bounded by the exchange limit of moe_b200_set_wait_limits (device error
 * MOE_DERR_TIMEOUT_FULL). Every GPU must make the same sequence of calls.
 * Workspace: moe_b200_layer_workspace_size(layer, world) bytes, zero-filled
 * once. Gate and up share a type; the type pair needs a fused kernel
 * (moe_b200_layer_fused(layer, world)); world <= 8. */
size_t moe_b200_ep_decode_buffer_bytes(int64_t H, int64_t n_experts_global, int64_t k, int32_t world);
int moe_b200_ep_layer_decode_p2p(const moe_layer_desc *layer, int64_t expert_lo, int64_t n_experts_global,
                                 const void *const *peer_bufs, int32_t world, int32_t rank, const float *x,
                                 const float *logits, float *out, void *workspace, size_t workspace_bytes,
                                 moe_stream_t stream);

/* No counterpart in the reference: 1 when moe_b200_layer_decode runs this
 * layer as one fused kernel for n_tok tokens (gate/up and down type pair with a
 * fused kernel, n_tok <= 8, n_tok * k <= 64, activations and tiles fit in
 * shared memory, fusion enabled), else 0. */
int moe_b200_layer_fused(const moe_layer_desc *layer, int64_t n_tok);

/* No counterpart in the reference: which kernel moe_b200_layer_decode runs
 * for fusable layers. 1 (the default): one launch with the grid cut into
 * per-expert CTA groups (h exchanged inside a group, output rows summed by
 * the CTA that completes them). 2: one launch where every CTA computes all
 * picks' down rows of its own output slice after a grid-wide exchange of h.
 * 0: four launches (routing, gate/up GEMV, down GEMV, combine). All three
 * give the same bits. GGML_CUDA_MOE_LAYER_FUSED=0/1/2 sets it at start-up. */
int moe_b200_layer_set_fused(int32_t enable);

/* No counterpart in the reference. A layer decode for callers that cannot
 * allocate device memory where they run it: engines that reserve all device
 * memory at start-up and own every byte, plugins whose host framework forbids
 * allocations inside its compute callback, or loops that must not take the
 * implicit synchronisation an allocation can cause. Same kernels and result as
 * moe_b200_layer_decode, but every piece of scratch (routing ids and weights,
 * GLU outputs, per-pick down outputs, expert pointer tables, an error word)
 * lives in one fixed file-scope device array of about 2.3 MB that every GPU
 * loading the library holds until exit; nothing is allocated and the
 * hot-expert cache is not used (expert tensors must be in device memory; no
 * stamps or hit/miss bookkeeping). Limits: n_tok <= 8, k <= 8, H <= 4096,
 * F <= 4096, n_experts <= 1024; larger requests return MOE_ERR_UNSUPPORTED.
 * Gate and up must share one type and shape (else MOE_ERR_INVALID); the
 * shared expert, when present, is read with the routed tensors' types.
 * The first call on a device looks up the array's address (cudaGetSymbolAddress)
 * and should come before any stream capture. All calls share the array and it
 * keeps the last call's contents, so calls that overlap on the GPU race. */
int moe_b200_layer_decode_noalloc(const moe_layer_desc *layer, const float *x, const float *logits, float *out,
                                  int64_t n_tok, moe_stream_t stream);

/* No counterpart in the reference: synchronise `stream`, then read the
 * moe_b200_layer_decode_noalloc device error word (0 = none; cleared by each
 * no-alloc call). */
int moe_b200_noalloc_device_error(moe_stream_t stream, int32_t *code);

/* No counterpart in the reference: synthetic weights for tests and benches:
 * n_rows rows of n_cols values ~ N(0, sigma) from a counter-based hash of
 * (seed, element index), quantized on the device with this project's min/max
 * quantizer (the same algorithm as the CPU oracle's). */
int moe_b200_fill_quantized(int32_t type, void *dst, int64_t n_rows, int64_t n_cols, uint64_t seed,
                            float sigma, moe_stream_t stream);

#ifdef __cplusplus
}
#endif
