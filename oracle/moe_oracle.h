/*
 * moe_oracle.h -- CPU restatement of the reference's MoE MUL_MAT_ID path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * product in a6000-custom-kernels_b200/. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference legs may load it. The product never
 * links or calls it.
 *
 * What it restates (all paths inside the reference project unless noted):
 *   - ggml_compute_forward_mul_mat_id and its _one_chunk worker
 *     (patches/trace-hook/ggml-cpu.c:1492-1553, 1563-1767): quantize src1 to
 *     the weight type's vec_dot_type, group (pick, token) rows by expert,
 *     one vec_dot per output element, dst[token][pick][row].
 *   - the CPU type-traits pairing (ggml-cpu.c:250-339): Q4_0/Q5_0/Q8_0 with
 *     Q8_0 activations, Q2_K..Q6_K with Q8_K activations.
 *   - the per-type vec_dot kernels and the Q8_0 / Q8_K activation quantizers,
 *     which live in llama.cpp @ 11fe0215 ggml-cpu/quants.c and ggml-quants.c.
 *     That third-party code is NOT present in the reference tree; these are
 *     restated from llama.cpp's published generic (non-SIMD) algorithms.
 *   - the Q8_1 activation format as produced by llama.cpp's CUDA quantize_q8_1
 *     (the input of the reference kernel, kernels/moe-cache.cu:206), and an
 *     exact (double precision) dot in that mode.
 *
 * Parity pinning: block decoding of all eight weight formats and the Q4_0 /
 * Q5_0 / Q8_0 quantizers are pinned against gguf-py 0.19.0 (an independent
 * implementation of the same formats) through tests/golden/. The vec_dot and
 * MUL_MAT_ID arithmetic has no golden vector in the reference (it ships no
 * tests), so that part is unpinned.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type numbering */
enum {
    ORC_F32 = 0, ORC_F16 = 1,
    ORC_Q4_0 = 2, ORC_Q5_0 = 6, ORC_Q8_0 = 8, ORC_Q8_1 = 9,
    ORC_Q2_K = 10, ORC_Q3_K = 11, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14,
    ORC_Q8_K = 15,
};

/* GLU ops, same numbering as the product's MOE_GLU_* */
enum { ORC_GLU_SWIGLU = 0, ORC_GLU_GEGLU = 1, ORC_GLU_SWIGLU_OAI = 2,
       ORC_GLU_SWIGLU_CLAMP = 3, ORC_GLU_PRODUCT = 4 };

int      orc_blck_size(int type);
int      orc_type_size(int type);
size_t   orc_row_size(int type, int64_t n);
uint16_t orc_fp32_to_fp16(float f);
float    orc_fp16_to_fp32(uint16_t h);
int      orc_vec_dot_type(int type);

int orc_dequantize_row(int type, const void *src, float *dst, int64_t n);
/* weight quantizer (synthetic data): Q4_0/Q5_0/Q8_0 follow ggml's reference
 * quantizers; K-quants use this project's min/max quantizer (format-exact) */
int orc_quantize_row(int type, const float *src, void *dst, int64_t n);
/* activation quantizers: ORC_Q8_0 (quantize_row_q8_0_ref), ORC_Q8_K
 * (quantize_row_q8_K_ref), ORC_Q8_1 (CUDA quantize_q8_1 semantics) */
int orc_quantize_act(int act_type, const float *src, void *dst, int64_t n);

/* one dot product of a weight row with an activation row.
 * exact == 0: llama.cpp generic CPU arithmetic (act_type must equal
 *             orc_vec_dot_type(type)).
 * exact == 1: exact value in double of sum(w_dequant * a_dequant) for any
 *             act_type in {Q8_0, Q8_1, Q8_K}. */
int orc_vec_dot(int type, int act_type, int exact, int64_t n,
                const void *w, const void *a, float *out);

/* MUL_MAT_ID restated from ggml-cpu.c:1563-1767.
 *   experts[e] -> base of expert e ([rows][row_bytes])
 *   src1  f32 [n_tok][ne11][K]  (ne11 == 1 broadcasts one row to all picks)
 *   ids   i32 [n_tok][n_used]
 *   dst   f32 [n_tok][n_used][rows]
 * act_type: activation format used for the dots (normally the CPU pairing). */
int orc_mul_mat_id(int type, int act_type, int exact,
                   const void *const *experts, int64_t n_experts,
                   int64_t K, int64_t rows, size_t row_bytes,
                   const float *src1, int64_t ne11, int64_t n_tok,
                   const int32_t *ids, int64_t n_used,
                   float *dst, int n_threads);

/* the same MUL_MAT_ID with an already-quantized Q8_1 src1 (the exact input of
 * the reference GPU kernel): src1_q8_1 is [n_tok][ne11][K/32] blocks of 36 B */
int orc_mul_mat_id_q8_1(int type, const void *const *experts, int64_t n_experts,
                        int64_t K, int64_t rows, size_t row_bytes,
                        const void *src1_q8_1, int64_t ne11, int64_t n_tok,
                        const int32_t *ids, int64_t n_used,
                        float *dst, int n_threads);

float orc_glu(int op, float gate, float up, float limit);

/* routing: top-k on logits (descending, ties -> lower index), weights =
 * softmax(logits)[selected], optionally renormalised over the k picks */
int orc_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts,
                     int64_t k, int norm_w, int32_t *ids, float *weights);

typedef struct {
    int          type_gate, type_up, type_down;
    const void *const *gate;   /* [n_experts] -> [F][H] */
    const void *const *up;     /* [n_experts] -> [F][H] */
    const void *const *down;   /* [n_experts] -> [H][F] */
    int          shared_type;  /* -1: none; else present, with the routed tensors' types */
    const void  *shared_gate, *shared_up, *shared_down;
    int64_t      H, F, n_experts, k;
    int          glu_op;
    float        glu_limit;
    int          norm_w;
} orc_layer;

/* One MoE FFN layer (llama.cpp build_moe_ffn order): route, gate/up
 * MUL_MAT_ID, GLU, down MUL_MAT_ID, weighted sum over picks in pick order,
 * plus the shared expert. act_mode: 0 = CPU pairing (Q8_0/Q8_K), 1 = Q8_1.
 * exact: see orc_vec_dot. out f32 [n_tok][H]. */
int orc_moe_layer(const orc_layer *L, const float *x, const float *logits,
                  int64_t n_tok, int act_mode, int exact, float *out,
                  int32_t *ids_out, float *w_out, int n_threads);

/* synthetic weights: rows [row0, row0 + n_rows) of a matrix of n_cols
 * columns, element (r, c) ~ N(0, sigma) from a counter hash of (seed,
 * r*n_cols + c) with Box-Muller (the device generator's recipe; libm may differ
 * by an ulp), quantized with orc_quantize_row. dst gets n_rows rows. */
int orc_fill_quantized(int type, void *dst, int64_t row0, int64_t n_rows, int64_t n_cols, uint64_t seed,
                       float sigma, int n_threads);

#ifdef __cplusplus
}
#endif
