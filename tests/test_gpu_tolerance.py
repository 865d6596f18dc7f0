"""End-to-end error of the batch-1 layer decode against the oracle (llama.cpp's
CPU MUL_MAT_ID in its MoE graph order) over many tokens, for the BASELINE
configs 1, 2 and 3 (two of config 3's per-tensor type draws). Every token is
held to layer_check's policy -- 1e-3 of its max |ref|, or a near-tie in the
re-quantized h and 1e-2 -- and the distribution is printed (pytest -s):
median, 99th percentile and maximum per-token error, and how many tokens had
a near-tie in h."""
import numpy as np
import pytest
import torch

import oracle as O
from layer_check import LAYER_TOL, check_layer
from moe_data import activations, zipf_logits

pytestmark = pytest.mark.gpu

N_TOK = 48
CASES = [
    # name, H, F, E, (gate, up, down), shared expert, Zipf routing
    ("config1", 2048, 512, 64, (O.Q4_0, O.Q4_0, O.Q4_0), False, False),
    ("config2", 3072, 768, 512, (O.Q2_K, O.Q2_K, O.Q2_K), True, True),
    ("config3 Q3_K/Q3_K/Q6_K", 3072, 768, 512, (O.Q3_K, O.Q3_K, O.Q6_K), True, True),
    ("config3 Q4_K/Q4_K/Q2_K", 3072, 768, 512, (O.Q4_K, O.Q4_K, O.Q2_K), True, True),
]


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    yield
    pkg.moe_cache.reset()


@pytest.mark.parametrize("name,H,F,E,types,shared,zipf", CASES, ids=[c[0] for c in CASES])
def test_layer_error_distribution(pkg, cuda, name, H, F, E, types, shared, zipf):
    k = 8
    layer = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=shared, seed=17)
    L = dict(H=H, F=F, E=E, k=k, type_gate=types[0], type_up=types[1], type_down=types[2])
    for r in ("gate", "up", "down"):
        L[r] = layer.w[r].cpu().numpy()
        if shared:
            L["shared_" + r] = layer.shared[r].cpu().numpy()
    if shared:
        L["shared_type"] = types[1]
    errs, ties = [], 0
    for i in range(N_TOK):
        x = activations((1, H), seed=1000 + i)
        logits = zipf_logits(1, E, seed=2000 + i) if zipf else activations((1, E), seed=2000 + i)
        out = layer.decode(torch.from_numpy(x).to(cuda), torch.from_numpy(logits).to(cuda)).cpu().numpy()
        assert pkg.moe_cache.device_error() == 0
        e = check_layer(layer, L, x, logits, out)
        errs.append(float(e["per_token"][0]))
        ties += int(e["requant_bytes_differing"][0] > 0)
    errs = np.array(errs)
    print(f"\n{name}: per-token max rel err over {N_TOK} tokens: median {np.median(errs):.2e}, "
          f"p99 {np.quantile(errs, 0.99):.2e}, max {errs.max():.2e}; tokens over {LAYER_TOL:g}: "
          f"{int((errs >= LAYER_TOL).sum())}; tokens with a near-tie in h: {ties}")
