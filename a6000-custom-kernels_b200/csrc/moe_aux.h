// moe_aux.h -- launchers of the small kernels around the GEMV (moe_aux.cu)
// and of the GEMV itself (moe_gemv.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

struct GemvArgs;
struct LayerArgs;
struct Layer2Args;
struct StackArgs;
struct MmqArgs;

cudaError_t launch_quantize_act(int act_type, const float *x, void *y, int64_t n_rows, int64_t n_cols,
                                cudaStream_t st);
cudaError_t launch_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts, int64_t k, int norm_w,
                                int32_t *ids, float *weights, cudaStream_t st);
// u[i] = GLU(op, g[i], u[i]) for i < n (the fused epilogue's glu_apply)
cudaError_t launch_glu(const float *g, float *u, int64_t n, int op, float limit, cudaStream_t st);
// out[t][r] = sum over the picks p with ids[t][p] in [id_lo, id_lo + n_local)
// of w * y (pick order), plus ys; 0 + ys when no pick is local
cudaError_t launch_combine_local(const float *y, const float *w, const float *ys, const int32_t *ids, int id_lo,
                                 int n_local, float *out, int64_t n_tok, int64_t H, int64_t k, cudaStream_t st);
cudaError_t launch_combine(const float *y, const float *w, const float *ys, float *out, int64_t n_tok, int64_t H,
                           int64_t k, cudaStream_t st);
cudaError_t launch_fill_quantized(int type, void *dst, int64_t n_rows, int64_t n_cols, uint64_t seed, float sigma,
                                  cudaStream_t st);

// Plans the launch geometry into `a` and launches the GEMV for weight type
// `type` with activation semantics `act`. Returns 0, or a negative MOE_ERR_*
// with *why set, or MOE_ERR_CUDA with *cuda_err set.
int launch_gemv(int type, int act, GemvArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err);

// Fused layer kernel (moe_layer.cu) for gate/up type ta and down type tb:
// plan_layer fills the geometry of `a` and returns 0 when the fused kernel
// handles the layer, else -2 with *why; launch_layer plans and launches
// (-3 with *cuda_err on a CUDA error).
int plan_layer(int ta, int tb, LayerArgs &a, int *grid, size_t *smem, const char **why);
int launch_layer(int ta, int tb, LayerArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err);
// The per-expert-group layer kernel (moe_layer2.cuh), same contract.
int plan_layer2(int ta, int tb, Layer2Args &a, int *grid, size_t *smem, const char **why);
int launch_layer2(int ta, int tb, Layer2Args &a, cudaStream_t st, const char **why, cudaError_t *cuda_err);
// The persistent stack kernel (moe_stack.cuh) for layers of one type.
bool stack_type_supported(int ta, int tb);
int launch_stack(int type, StackArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err);
// The mixed-type stack kernel: each layer's gate/up and down types among
// Q2_K, Q3_K, Q4_K, Q6_K (StackLayer::ta / tb = their slots); used_a / used_b
// = bit masks of the slots in use (the stages are sized for the largest).
bool stack_mix_supported(int type);
int launch_stack_mixed(unsigned used_a, unsigned used_b, StackArgs &a, cudaStream_t st, const char **why,
                       cudaError_t *cuda_err);

// Prefill grouped GEMM on the tensor cores (moe_mmq.cu): launch_mmq_group
// groups the (token, pick) entries by expert into offsets / entries and the
// tile prefix; launch_mmq runs the int8 MMQ over that tile list (-2 with *why
// when the type or shape has no tensor-core path, -3 with *cuda_err).
cudaError_t launch_mmq_group(const int32_t *ids, int64_t ids_stride, int n_tok, int k, int E, int ntc,
                             int32_t *entries, int4 *chunks, int32_t *n_chunks, int *err, cudaStream_t st,
                             bool skip_empty = false);
// B tiles quantized from f32 rows x [rows][K] (one row per entry), or from
// GLU(op, x, u) when u is set
cudaError_t launch_mmq_gather_rows(const float *x, const float *u, int glu_op, float glu_limit, int K,
                                   const int32_t *entries, const int4 *chunks, const int32_t *n_chunks, int ntc,
                                   int64_t max_chunks, uint8_t *btiles, cudaStream_t st);
// launch_mmq_gather writes the chunks' B tiles (MMQ layout) from the tokens'
// Q8_K rows x8 [n_tok][K / 256]; max_chunks bounds the chunk count
// (mmq_max_chunks).
cudaError_t launch_mmq_gather(const uint8_t *x8, int K, int k, int ntc, const int32_t *entries, const int4 *chunks,
                              const int32_t *n_chunks, int64_t max_chunks, uint8_t *btiles, cudaStream_t st);
// Expert-parallel exchange over peer memory (moe_ep.cu). peer_ptrs: [5][W]
// device pointers as seen from this GPU (received rows, their ids, their
// source entries, returned outputs, arrival counters) of every GPU; scratch:
// 16 zeroed uint32 per GPU (cursors and block counters, reset after use).
cudaError_t launch_ep_dispatch(const void *const *peer_ptrs, int W, int me, int cap, const int32_t *ids,
                               int n_entries, int k, int E, const float *x, int H, uint32_t *scratch, int *err,
                               cudaStream_t st);
cudaError_t launch_ep_return(const void *const *peer_ptrs, int W, int cap, const int32_t *ids, const int32_t *src,
                             const float *y, int H, uint32_t *scratch, cudaStream_t st);
cudaError_t launch_ep_wait(const uint32_t *flag, uint32_t target, uint64_t timeout_ns, int *err, cudaStream_t st);

// chunk table of a one-expert call with all ids 0: entries in order, chunks
// of ntc consecutive entries
cudaError_t launch_mmq_identity_chunks(int n, int ntc, int32_t *entries, int4 *chunks, int32_t *n_chunks,
                                       cudaStream_t st);

// tokens per chunk of the tensor-core path for a weight type (0: none)
int mmq_chunk_tokens(int type);
bool mmq_supported(int type, int64_t K, int64_t nrows);
cudaError_t launch_mmq_pool_ids(const int32_t *ids, int64_t ids_stride, int n_tok, int k, char *const *tbl,
                                int n_experts, const char *pool, uint64_t expert_bytes, int n_slots, int32_t *out,
                                cudaStream_t st);
bool mmq_b32(int type);              // Q4_0 / Q5_0 / Q8_0: 32-weight blocks, Q8_0 activations
int mmq_step(int type);              // weights per row and MMQ step (256, or 128 for Q8_0)
uint32_t mmq_bt_stride(int type);    // bytes between B tiles
cudaError_t launch_mmq_gather32(const uint8_t *x8, int K, int sk, int k, int ntc, const int32_t *entries,
                                const int4 *chunks, const int32_t *n_chunks, int64_t max_chunks, uint8_t *btiles,
                                uint32_t bt_stride, cudaStream_t st);
int launch_mmq(int type, MmqArgs &a, cudaStream_t st, const char **why, cudaError_t *cuda_err);

}  // namespace moe
