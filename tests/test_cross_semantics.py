"""The gap between llama.cpp's two activation semantics for MUL_MAT_ID: the
CUDA MMVQ path (Q8_1 activations, what the reference kernel consumes) and the
CPU path (Q8_K / Q8_0 activations, the parity target). Both sides here are
the oracle, so this pins the size of the gap itself: every output lies
within 6 sigma of the rounding model in moe_data.act_quant_sigma, and the
worst output relative to max |ref| is what the GPU cross-check
(tests/test_gpu_gemv.py) can at most add to its own tight error."""
import numpy as np
import pytest

import oracle as O
from moe_data import act_quant_sigma, activations, distinct_ids, experts, rel_err

Z_MAX = 6.0


@pytest.mark.parametrize("t", O.WEIGHT_TYPES)
def test_activation_semantics_gap_is_rounding_noise(t):
    E, rows, K, n_tok, n_used = 8, 128, 1024, 2, 4
    W = experts(t, E, rows, K, seed=1)
    ids = distinct_ids(n_tok, n_used, E, seed=2)
    x = activations((n_tok, 1, K), seed=3)
    q81 = O.mul_mat_id_q8_1(t, W, K, O.quantize_act(O.Q8_1, x), ids)
    cpu = O.mul_mat_id(t, W, K, x, ids, exact=0)
    sigma = act_quant_sigma(t, W, K, x[:, 0], ids)
    z = np.abs(q81.astype(np.float64) - cpu) / sigma
    print(f"{O.TYPE_NAMES[t]}: gap rel err {rel_err(q81, cpu):.2e}, max |gap| / sigma {z.max():.2f}, "
          f"mean {z.mean():.2f}")
    assert z.max() < Z_MAX
