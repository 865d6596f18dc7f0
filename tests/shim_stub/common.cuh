// Test stand-in for llama.cpp's ggml-cuda/common.cuh: only the declarations
// the libmoe_b200 adapter (a6000-custom-kernels_b200/shim/moe-cache.cu)
// touches, with the member names and types it reads. Used to check that the
// adapter compiles and links; it is not llama.cpp.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q2_K = 10 };

enum ggml_glu_op {
    GGML_GLU_OP_REGLU,
    GGML_GLU_OP_GEGLU,
    GGML_GLU_OP_SWIGLU,
    GGML_GLU_OP_SWIGLU_OAI,
    GGML_GLU_OP_GEGLU_ERF,
    GGML_GLU_OP_GEGLU_QUICK,
    GGML_GLU_OP_SWIGLU_CLAMP,
};

struct ggml_backend_buffer;

struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer * buffer;
    int64_t ne[4];
    size_t nb[4];
    struct ggml_tensor * view_src;
    void * data;
    char name[64];
};

struct ggml_backend_cuda_context {
    int device;
};

struct ggml_cuda_mm_fusion_args_host {
    const ggml_tensor * gate;
};

struct ggml_cuda_mm_fusion_args_device {
    const void * gate;
    const void * x_bias;
    const void * gate_bias;
    const void * x_scale;
    const void * gate_scale;
    ggml_glu_op glu_op;
    float glu_limit;
    const void * shared_up;
    const void * shared_gate;
    float * shared_dst;
    int64_t shared_stride_col_dst;
};

#define GGML_UNUSED(x) (void) (x)
#define GGML_ABORT(...)                   \
    do {                                  \
        fprintf(stderr, __VA_ARGS__);     \
        fputc('\n', stderr);              \
        abort();                          \
    } while (0)
