// moe-cache.cu -- llama.cpp adapter onto libmoe_b200.so. Each function
// converts the ggml arguments to the C ABI's plain descriptors and calls the
// C entry point of the same name. The C declarations are read inside
// namespace mc: ggml_cuda_moe_cache_enabled(), _active() and _step() take the
// same parameters in both headers and differ only in the return type, which
// two declarations in one scope may not; in their own namespace the C
// functions (C linkage, plain symbol names) and these C++ definitions
// (mangled symbols) coexist. Errors abort through GGML_ABORT with the
// library's message, as the backend expects of this path.
#include <stddef.h>
#include <stdint.h>

#include "moe-cache.cuh"

namespace mc {
#include "moe_cache_b200.h"
}

namespace {

using mc::moe_tensor;

moe_tensor describe(const ggml_tensor * t) {
    moe_tensor d = {};
    d.data = t->data;
    d.type = static_cast<int32_t>(t->type);           // ggml_type ids are the C ABI's type ids
    d.flags = (t->view_src ? MOE_TENSOR_VIEW : 0) | (t->buffer ? 0 : MOE_TENSOR_NO_BUFFER);
    for (int i = 0; i < 4; ++i) {
        d.ne[i] = t->ne[i];
        d.nb[i] = static_cast<uint64_t>(t->nb[i]);
    }
    d.name = t->name;
    return d;
}

int32_t glu_of(ggml_glu_op op) {
    switch (op) {
        case GGML_GLU_OP_SWIGLU:       return mc::MOE_GLU_SWIGLU;
        case GGML_GLU_OP_GEGLU:        return mc::MOE_GLU_GEGLU;
        case GGML_GLU_OP_SWIGLU_OAI:   return mc::MOE_GLU_SWIGLU_OAI;
        case GGML_GLU_OP_SWIGLU_CLAMP: return mc::MOE_GLU_SWIGLU_CLAMP;
        default:                       return mc::MOE_GLU_PRODUCT;
    }
}

void require(int rc, const char * what) {
    if (rc != MOE_OK) {
        GGML_ABORT("moe-cache: %s failed: %s", what, mc::moe_b200_last_error());
    }
}

}  // namespace

bool ggml_cuda_moe_cache_enabled() { return mc::ggml_cuda_moe_cache_enabled() != 0; }

bool ggml_cuda_moe_cache_active() { return mc::ggml_cuda_moe_cache_active() != 0; }

bool ggml_cuda_moe_cache_wants(const ggml_tensor * src0) {
    const moe_tensor d = describe(src0);
    return mc::ggml_cuda_moe_cache_wants(&d) != 0;
}

bool ggml_cuda_moe_cache_pin_host(const ggml_tensor * t) {
    const moe_tensor d = describe(t);
    return mc::ggml_cuda_moe_cache_pin_host(&d) != 0;
}

void ggml_cuda_moe_cache_step(cudaStream_t stream) {
    require(mc::ggml_cuda_moe_cache_step(reinterpret_cast<mc::moe_stream_t>(stream)), "step");
}

void ggml_cuda_moe_cache_mul_mat_vec_q(
        ggml_backend_cuda_context & ctx,
        const ggml_tensor * src0, const ggml_tensor * ids, ggml_tensor * dst,
        const ggml_cuda_mm_fusion_args_host * fusion, const ggml_cuda_mm_fusion_args_device & fusion_dev,
        const char * src1_q8_1, const int32_t * ids_d, float * dst_d,
        int64_t ne00, int64_t ne01, int64_t ne02, int64_t ne03,
        int64_t ncols_dst, int64_t s01, int64_t s02, int64_t s03,
        int64_t nchannels_y, int64_t nchannels_dst,
        int64_t stride_col_y, int64_t stride_col_dst,
        int64_t stride_channel_y, int64_t stride_channel_dst,
        int64_t ids_stride, cudaStream_t stream) {
    GGML_UNUSED(ctx);
    GGML_UNUSED(ids);
    GGML_UNUSED(dst);
    const moe_tensor experts = describe(src0);
    moe_tensor gate;
    mc::moe_fusion_host host = {};
    if (fusion && fusion->gate) {
        gate = describe(fusion->gate);
        host.gate = &gate;
    }
    mc::moe_fusion_device dev = {};
    dev.gate = fusion_dev.gate;
    dev.x_bias = static_cast<const float *>(fusion_dev.x_bias);
    dev.gate_bias = static_cast<const float *>(fusion_dev.gate_bias);
    dev.x_scale = static_cast<const float *>(fusion_dev.x_scale);
    dev.gate_scale = static_cast<const float *>(fusion_dev.gate_scale);
    dev.glu_op = glu_of(fusion_dev.glu_op);
    dev.glu_limit = fusion_dev.glu_limit;
    dev.shared_up = fusion_dev.shared_up;
    dev.shared_gate = fusion_dev.shared_gate;
    dev.shared_dst = fusion_dev.shared_dst;
    dev.shared_stride_col_dst = fusion_dev.shared_stride_col_dst;
    require(mc::ggml_cuda_moe_cache_mul_mat_vec_q(
                &experts, &host, &dev, src1_q8_1, mc::MOE_TYPE_Q8_1, ids_d, dst_d, ne00, ne01, ne02, ne03, ncols_dst,
                s01, s02, s03, nchannels_y, nchannels_dst, stride_col_y, stride_col_dst, stride_channel_y,
                stride_channel_dst, ids_stride, reinterpret_cast<mc::moe_stream_t>(stream)),
            "MUL_MAT_ID");
}
