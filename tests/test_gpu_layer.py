"""A full MoE layer (route, fused gate/up + SwiGLU + shared expert, down,
weighted combine) on the GPU against the oracle's llama.cpp-order layer, stage
by stage (tests/layer_check.py): routing ids bit-exact, every stage within
1e-4 of max |ref|, the end-to-end output within 1e-2."""
import numpy as np
import pytest
import torch

import oracle as O
from layer_check import check_layer
from moe_data import activations, experts, zipf_logits

pytestmark = pytest.mark.gpu


def _layer_np(types, H, F, E, seed):
    tg, tu, td = types
    return dict(H=H, F=F, E=E, type_gate=tg, type_up=tu, type_down=td,
                gate=experts(tg, E, F, H, seed), up=experts(tu, E, F, H, seed + 1), down=experts(td, E, H, F, seed + 2),
                shared_type=tu, shared_gate=experts(tg, 1, F, H, seed + 3)[0], shared_up=experts(tu, 1, F, H, seed + 4)[0],
                shared_down=experts(td, 1, H, F, seed + 5)[0])


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    yield
    pkg.moe_cache.reset()


@pytest.mark.parametrize("types,n_tok", [((O.Q2_K, O.Q2_K, O.Q2_K), 1), ((O.Q3_K, O.Q3_K, O.Q6_K), 4),
                                         ((O.Q4_K, O.Q4_K, O.Q5_K), 8), ((O.Q4_0, O.Q4_0, O.Q8_0), 2),
                                         ((O.Q5_0, O.Q5_0, O.Q4_0), 1),
                                         # gate and up of different types: two GEMVs and a GLU pass
                                         ((O.Q2_K, O.Q4_K, O.Q3_K), 1), ((O.Q6_K, O.Q3_K, O.Q2_K), 5)])
def test_layer_decode_matches_oracle(pkg, cuda, types, n_tok):
    H, F, E, k = 1024, 512, 24, 8
    L = _layer_np(types, H, F, E, seed=sum(types))
    L["k"] = k
    x = activations((n_tok, H), seed=1)
    logits = zipf_logits(n_tok, E, seed=2)
    layer = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=True,
                         weights={r: L[r] for r in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down")})
    out = layer.decode(torch.from_numpy(x).to(cuda), torch.from_numpy(logits).to(cuda))
    assert pkg.moe_cache.device_error() == 0
    check_layer(layer, L, x, logits, out.cpu().numpy())


def test_config2_layer_full_expert_count(pkg, cuda):
    """Config 2: H=3072, F=768, 512 experts, top-8 Zipf routing, shared expert,
    Q2_K; weights from the device generator, checked for the routed experts."""
    H, F, E, k, n_tok = 3072, 768, 512, 8, 2
    layer = pkg.MoELayer(H, F, E, k, {"gate": O.Q2_K, "up": O.Q2_K, "down": O.Q2_K}, shared=True, seed=3)
    x = activations((n_tok, H), seed=4)
    logits = zipf_logits(n_tok, E, seed=5)
    out = layer.decode(torch.from_numpy(x).to(cuda), torch.from_numpy(logits).to(cuda)).cpu().numpy()
    L = dict(H=H, F=F, E=E, k=k, type_gate=O.Q2_K, type_up=O.Q2_K, type_down=O.Q2_K, shared_type=O.Q2_K)
    for r in ("gate", "up", "down"):
        L[r] = layer.w[r].cpu().numpy()
        L["shared_" + r] = layer.shared[r].cpu().numpy()
    check_layer(layer, L, x, logits, out)


def test_decode_trace_builds_seed(pkg, cuda, tmp_path):
    """decode steps traced in the trace hook's format give a seed file whose
    lines start with the most picked experts of each tensor"""
    from importlib import import_module
    S = import_module("a6000-custom-kernels_b200.seed")
    H, F, E, k = 1024, 512, 24, 8
    layer = pkg.MoELayer(H, F, E, k, {"gate": O.Q2_K, "up": O.Q2_K, "down": O.Q2_K}, shared=False, seed=5,
                         name="blk.3")
    path = tmp_path / "trace.bin"
    picks = {}
    with S.TraceWriter(str(path)) as w:
        for step in range(12):
            x = torch.from_numpy(activations((1, H), seed=100 + step)).to(cuda)
            lg = torch.from_numpy(zipf_logits(1, E, seed=200 + step)).to(cuda)
            layer.decode(x, lg, trace=w)
            for e in layer.routing_of(1)[0].cpu().numpy().reshape(-1).tolist():
                picks[e] = picks.get(e, 0) + 1
    order = S.build_seed(str(path), str(tmp_path / "seed.txt"))
    assert list(order) == [f"blk.3.ffn_{r}_exps.weight" for r in ("gate", "up", "down")]
    top = max(picks.values())
    assert picks[order["blk.3.ffn_gate_exps.weight"][0]] == top
    assert sorted(order["blk.3.ffn_down_exps.weight"]) == sorted(picks)
