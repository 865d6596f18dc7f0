"""Self-consistency of the CPU oracle: llama.cpp-arithmetic dots against exact
dots, MUL_MAT_ID grouping against a direct numpy evaluation, activation
quantizer properties, GLU and routing."""
import numpy as np
import pytest

import oracle as O
from moe_data import activations, distinct_ids, experts, rel_err, zipf_logits


@pytest.mark.parametrize("t", O.WEIGHT_TYPES)
def test_generic_dot_close_to_exact(t):
    K = 512
    w = experts(t, 1, 8, K, seed=t)[0]
    x = activations((K,), seed=100 + t)
    at = O.vec_dot_type(t)
    a = O.quantize_act(at, x)
    for r in range(8):
        g = O.vec_dot(t, at, 0, w[r], a, K)
        e = O.vec_dot(t, at, 1, w[r], a, K)
        assert abs(g - e) <= 1e-5 * max(1.0, abs(e)) + 1e-6


@pytest.mark.parametrize("t", O.WEIGHT_TYPES)
def test_exact_dot_equals_dequantized_product(t):
    """Exact mode = sum(w * a) of the dequantized values -- except Q4_0 / Q5_0
    with Q8_1 activations, where llama.cpp's CUDA dot takes the weights'
    offset off with the block's stored s (f16 sum of the unquantized x):
    sum(w * a) + offset * sum over blocks of d_w (sum(a) - s)."""
    K = 256
    w = experts(t, 1, 4, K, seed=7)[0]
    x = activations((K,), seed=8)
    off = {O.Q4_0: 8, O.Q5_0: 16}.get(t, 0)
    for at in (O.Q8_0, O.Q8_1, O.Q8_K):
        a = O.quantize_act(at, x)
        wd = O.dequantize(t, w, 4 * K).reshape(4, K).astype(np.float64)
        ad = O.dequantize(at, a, K).reshape(K).astype(np.float64)
        for r in range(4):
            e = O.vec_dot(t, at, 1, w[r], a, K)
            ref = float(wd[r] @ ad)
            if at == O.Q8_1 and off:
                dw = w[r].reshape(K // 32, -1)[:, :2].copy().view(np.float16)[:, 0].astype(np.float64)
                s = a.reshape(K // 32, 36)[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float64)
                ref += off * float((dw * (ad.reshape(K // 32, 32).sum(axis=1) - s)).sum())
            assert abs(e - ref) <= 2e-4 * max(1.0, abs(ref))


def test_q8_K_quantizer_properties():
    x = activations((4, 512), seed=3)
    x[1, :256] = 0.0
    x[2, 10] = -50.0
    q = O.quantize_act(O.Q8_K, x).reshape(4, 2, 292)
    d = q[..., :4].copy().view(np.float32)[..., 0]
    qs = q[..., 4:260].view(np.int8).astype(np.int32)
    bs = q[..., 260:292].copy().view(np.int16).astype(np.int32)
    np.testing.assert_array_equal(bs, qs.reshape(4, 2, 16, 16).sum(-1))
    assert d[1, 0] == 0 and (qs[1, 0] == 0).all()
    assert qs.min() >= -128 and qs.max() <= 127
    assert qs[2, 0, 10] == 127 or qs[2, 0, 10] == -127      # the extreme maps to +-127
    deq = O.dequantize(O.Q8_K, q.reshape(4, -1), 512 * 4).reshape(4, 512)
    assert np.abs(deq - x).max() <= np.abs(x).max() / 127 + 1e-6


def test_q8_1_quantizer_properties():
    x = activations((2, 64), seed=4)
    q = O.quantize_act(O.Q8_1, x).reshape(2, 2, 36)
    d = q[..., 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    s = q[..., 2:4].copy().view(np.float16).astype(np.float32)[..., 0]
    amax = np.abs(x.reshape(2, 2, 32)).max(-1)
    np.testing.assert_allclose(d, (amax / 127).astype(np.float16).astype(np.float32))
    np.testing.assert_allclose(s, x.reshape(2, 2, 32).sum(-1), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("t", [O.Q4_0, O.Q2_K, O.Q6_K])
@pytest.mark.parametrize("ne11", [1, 4])
def test_mul_mat_id_grouping(t, ne11):
    E, rows, K, n_tok, n_used = 6, 24, 256, 3, 4
    w = experts(t, E, rows, K, seed=11)
    ids = distinct_ids(n_tok, n_used, E, seed=12)
    ids[2, 1] = ids[0, 0]                      # shared expert across tokens
    src1 = activations((n_tok, ne11, K), seed=13)
    got = O.mul_mat_id(t, w, K, src1, ids, exact=1)
    at = O.vec_dot_type(t)
    wd = O.dequantize(t, w.reshape(E * rows, -1), E * rows * K).reshape(E, rows, K).astype(np.float64)
    for tok in range(n_tok):
        for p in range(n_used):
            a = O.quantize_act(at, src1[tok, p % ne11])
            ad = O.dequantize(at, a, K).reshape(K).astype(np.float64)
            ref = wd[ids[tok, p]] @ ad
            assert rel_err(got[tok, p], ref) < 1e-5


def test_mul_mat_id_q8_1_matches_exact_mode():
    t, E, rows, K = O.Q3_K, 4, 16, 512
    w = experts(t, E, rows, K, seed=5)
    ids = distinct_ids(2, 3, E, seed=6)
    x = activations((2, 1, K), seed=7)
    q = O.quantize_act(O.Q8_1, x)
    a = O.mul_mat_id(t, w, K, x, ids, act_t=O.Q8_1, exact=1)
    b = O.mul_mat_id_q8_1(t, w, K, q, ids)
    np.testing.assert_array_equal(a, b)


def test_glu_ops():
    g = np.array([-3.0, -0.5, 0.0, 0.7, 9.0], dtype=np.float32)
    u = np.array([1.0, -2.0, 3.0, 0.5, -9.0], dtype=np.float32)
    silu = g / (1 + np.exp(-g))
    np.testing.assert_allclose(O.glu(O.GLU_SWIGLU, g, u), u * silu, rtol=1e-6)
    np.testing.assert_allclose(O.glu(O.GLU_PRODUCT, g, u), u * g, rtol=1e-6)
    gel = 0.5 * g * (1 + np.tanh(0.7978845608 * g * (1 + 0.044715 * g * g)))
    np.testing.assert_allclose(O.glu(O.GLU_GEGLU, g, u), u * gel, rtol=1e-5, atol=1e-6)
    x = np.minimum(g, 7.0); uu = np.clip(u, -7, 7)
    np.testing.assert_allclose(O.glu(O.GLU_SWIGLU_OAI, g, u), x / (1 + np.exp(-1.702 * x)) * (uu + 1), rtol=1e-5)
    x = np.minimum(g, 2.0); uu = np.clip(u, -2, 2)
    np.testing.assert_allclose(O.glu(O.GLU_SWIGLU_CLAMP, g, u, 2.0), x / (1 + np.exp(-x)) * uu, rtol=1e-5)


def test_topk_softmax():
    logits = zipf_logits(5, 64, seed=9)
    logits[0, 3] = logits[0, 5] = 100.0        # a tie: lower id first
    ids, w = O.topk_softmax(logits, 8, norm_w=False)
    assert ids[0, 0] == 3 and ids[0, 1] == 5
    for t in range(5):
        order = sorted(range(64), key=lambda e: (-logits[t, e], e))[:8]
        assert list(ids[t]) == order
        p = np.exp(logits[t] - logits[t].max()); p /= p.sum()
        np.testing.assert_allclose(w[t], p[ids[t]], rtol=1e-5)
    _, wn = O.topk_softmax(logits, 8, norm_w=True)
    np.testing.assert_allclose(wn.sum(1), 1.0, rtol=1e-5)


def test_layer_matches_composition():
    H, F, E, k = 256, 256, 8, 2
    t = O.Q4_K
    layer = dict(H=H, F=F, E=E, k=k, type_gate=t, type_up=t, type_down=t,
                 gate=experts(t, E, F, H, 1), up=experts(t, E, F, H, 2), down=experts(t, E, H, F, 3),
                 shared_type=t, shared_gate=experts(t, 1, F, H, 4)[0], shared_up=experts(t, 1, F, H, 5)[0],
                 shared_down=experts(t, 1, H, F, 6)[0])
    x = activations((2, H), 7)
    logits = zipf_logits(2, E, 8)
    out, ids, w = O.moe_layer(layer, x, logits)
    g = O.mul_mat_id(t, layer["gate"], H, x[:, None], ids)
    u = O.mul_mat_id(t, layer["up"], H, x[:, None], ids)
    h = O.glu(O.GLU_SWIGLU, g, u)
    d = O.mul_mat_id(t, layer["down"], F, h, ids)
    z = np.zeros((2, 1), np.int32)
    sg = O.mul_mat_id(t, layer["shared_gate"][None], H, x[:, None], z)
    su = O.mul_mat_id(t, layer["shared_up"][None], H, x[:, None], z)
    sd = O.mul_mat_id(t, layer["shared_down"][None], F, O.glu(O.GLU_SWIGLU, sg, su), z)
    ref = (d * w[:, :, None]).sum(1) + sd[:, 0]
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)
