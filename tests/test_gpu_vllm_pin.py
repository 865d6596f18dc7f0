"""Pins the Q8_1-activation MUL_MAT_ID arithmetic -- the reference kernel's
own semantics: llama.cpp's CUDA vec_dot_*_q8_1 on activations quantized to
Q8_1 -- against an implementation that is not this project's: vLLM's port of
llama.cpp's MMVQ kernels for GGUF weights (`ggml_moe_a8_vec`, vLLM 0.22.0,
installed in this image as a library; used here only as a checker).

Both the oracle's Q8_1 path (orc_mul_mat_id_q8_1) and the GPU GEMV in Q8_1
mode are compared with it, on the same weight bytes and f32 activations, for
all eight weight types, in the gate/up form (one input per token, k picks)
and the down form (one input per pick). vLLM quantizes the f32 activations
to Q8_1 itself, so the comparison also covers the Q8_1 quantizer.

Tolerance: PIN = 1e-5 of max |ref| per output vector. The integer dot
products are exact on both sides; only the float steps (the per-block
d * sum terms and the order in which a row's partial sums are added) differ,
which at K = 1024 stays near f32 rounding (~1e-7 relative per add).
"""
import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, distinct_ids, experts, rel_err

pytestmark = pytest.mark.gpu

PIN = 1e-5


def _vllm_op():
    try:
        import vllm._custom_ops as ops
        op = ops.ggml_moe_a8_vec
        torch.ops._C.ggml_moe_a8_vec  # noqa: B018  (the compiled op is present)
    except Exception as e:  # vLLM absent or built without its CUDA ops
        pytest.skip(f"vLLM's GGUF MoE kernels are not available: {e}")
    return op


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    yield
    pkg.moe_cache.reset()


def _ours(pkg, cuda, t, W, K, rows, ids, src1):
    """The GEMV with Q8_1 activations (made by the oracle's quantizer, which is
    byte-exact with the kernel's): dst [n_tok][k][rows]."""
    mc = pkg.moe_cache
    n_tok, k = ids.shape
    nch = src1.shape[1]
    Wd = torch.from_numpy(W).to(cuda)
    src0 = mc.expert_tensor(Wd, t, K, rows, name="w")
    q = torch.from_numpy(O.quantize_act(O.Q8_1, src1)).to(cuda)
    ids_d = torch.from_numpy(ids).to(cuda)
    dst = torch.full((n_tok, k, rows), float("nan"), device=cuda)
    mc.mul_mat_vec_q(src0, q, mc.Q8_1, ids_d, dst, ncols_dst=n_tok, nchannels_y=nch, nchannels_dst=k,
                     stride_col_y=nch * (K // 32), stride_col_dst=k * rows, stride_channel_y=K // 32,
                     stride_channel_dst=rows, ids_stride=k)
    torch.cuda.synchronize()
    assert mc.device_error() == 0
    return dst.cpu().numpy()


@pytest.mark.parametrize("t", O.WEIGHT_TYPES)
@pytest.mark.parametrize("form", ["gate_up", "down"])
def test_q8_1_mul_mat_id_matches_vllm_port_of_llamacpp_mmvq(pkg, cuda, t, form):
    op = _vllm_op()
    E, rows, K, n_tok, k = 8, 256, 1024, 3, 4
    W = experts(t, E, rows, K, seed=60 + t)
    ids = distinct_ids(n_tok, k, E, seed=7)
    Wd = torch.from_numpy(W).to(cuda)
    if form == "gate_up":
        x = activations((n_tok, K), seed=8)
        got_v = op(torch.from_numpy(x).to(cuda), Wd, torch.from_numpy(ids).to(cuda), k, t, rows, n_tok)
        src1 = x[:, None, :]
    else:
        x = activations((n_tok, k, K), seed=9)
        got_v = op(torch.from_numpy(x.reshape(n_tok * k, K)).to(cuda), Wd,
                   torch.from_numpy(ids.reshape(n_tok * k, 1).copy()).to(cuda), 1, t, rows, n_tok * k)
        src1 = x
    torch.cuda.synchronize()
    v = got_v.float().cpu().numpy().reshape(n_tok, k, rows)
    ref = O.mul_mat_id_q8_1(t, W, K, O.quantize_act(O.Q8_1, src1), ids)
    ours = _ours(pkg, cuda, t, W, K, rows, ids, src1)
    e_oracle, e_gpu = rel_err(ref, v), rel_err(ours, v)
    print(f"\ntype {t} {form}: oracle vs vLLM {e_oracle:.2e}, GPU GEMV vs vLLM {e_gpu:.2e}")
    assert e_oracle < PIN, e_oracle
    assert e_gpu < PIN, e_gpu
