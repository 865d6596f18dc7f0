"""Bit-exact activation quantizers and routing ids, plus the synthetic-weight
generator, against the CPU oracle (through the C ABI)."""
import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, zipf_logits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act", [O.Q8_0, O.Q8_1, O.Q8_K])
def test_quantize_act_bit_exact(pkg, cuda, act):
    x = activations((7, 1024), seed=act)
    x[0, :256] = 0.0                          # all-zero blocks
    x[1, 17] = 40.0                           # a positive extreme
    x[2, 300] = -40.0                         # a negative extreme
    x[3, 5] = x[3, 6] = 9.0                   # tied maxima
    x[3, 7] = -9.0
    got = pkg.moe_cache.quantize_act(act, torch.from_numpy(x).to(cuda)).cpu().numpy()
    ref = O.quantize_act(act, x)
    np.testing.assert_array_equal(got, ref)


def test_topk_ids_bit_exact(pkg, cuda):
    for E, k, norm in ((512, 8, False), (64, 8, True), (128, 1, False), (40, 32, False)):
        logits = zipf_logits(9, E, seed=E + k)
        logits[0, 7] = logits[0, 9] = logits[0].max() + 1.0   # tie at the top
        ids, w = pkg.moe_cache.topk_softmax(torch.from_numpy(logits).to(cuda), k, norm_w=norm)
        rid, rw = O.topk_softmax(logits, k, norm_w=norm)
        np.testing.assert_array_equal(ids.cpu().numpy(), rid)
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("t", O.WEIGHT_TYPES)
def test_fill_quantized_is_valid_normal(pkg, cuda, t):
    rows, K = 64, 512
    buf = torch.empty((rows, O.row_size(t, K)), dtype=torch.uint8, device=cuda)
    pkg.moe_cache.fill_quantized(t, buf, rows, K, seed=5, sigma=0.02)
    w = O.dequantize(t, buf.cpu().numpy(), rows * K)
    assert np.isfinite(w).all()
    assert 0.014 < w.std() < 0.026 and abs(w.mean()) < 0.003
    buf2 = torch.empty_like(buf)
    pkg.moe_cache.fill_quantized(t, buf2, rows, K, seed=5, sigma=0.02)
    assert torch.equal(buf, buf2)
