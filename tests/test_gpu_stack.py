"""The persistent stack kernel (moe_b200_stack_prepare / _run): many batch-1
layers in one launch, each equal bit for bit to moe_b200_layer_decode of the
same layer and token -- as a residual chain (layer l + 1 reads x_l + out_l)
and with independent inputs, over repeated launches on one workspace."""
import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, zipf_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    yield
    pkg.moe_cache.reset()


@pytest.mark.parametrize("t,shape", [(O.Q2_K, (3072, 768, 64, 8)), (O.Q4_K, (1024, 512, 32, 4)),
                                     (O.Q4_0, (2048, 512, 64, 8))])
def test_stack_chain_equals_layer_by_layer(pkg, cuda, t, shape):
    H, F, E, k = shape
    n = 6
    layers = [pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, seed=50 + l) for l in range(n)]
    xs = [torch.zeros((1, H), device=cuda) for _ in range(n + 1)]
    xs[0].copy_(torch.from_numpy(activations((1, H), seed=3)))
    lgs = [torch.from_numpy(zipf_logits(1, E, seed=10 + l)).to(cuda) for l in range(n)]
    outs = [torch.zeros((1, H), device=cuda) for _ in range(n)]
    st = pkg.Stack(layers, xs[:n], lgs, outs, x_nexts=xs[1:])
    st.run()
    torch.cuda.synchronize()
    assert pkg.moe_cache.device_error() == 0
    x = xs[0].clone()
    for l in range(n):
        ref = layers[l].decode(x, lgs[l])
        assert torch.equal(outs[l], ref), l
        x = x + ref
        assert torch.equal(xs[l + 1], x), l
    # again on the same workspace: the same results
    first = [o.clone() for o in outs]
    st.run()
    torch.cuda.synchronize()
    for l in range(n):
        assert torch.equal(outs[l], first[l])


def test_stack_independent_inputs_cycle_layers(pkg, cuda):
    H, F, E, k = 3072, 768, 64, 8
    t = O.Q2_K
    layers = [pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, seed=70 + l) for l in range(2)]
    n = 20
    xs = [torch.from_numpy(activations((1, H), seed=100 + i)).to(cuda) for i in range(n)]
    lgs = [torch.from_numpy(zipf_logits(1, E, seed=200 + i)).to(cuda) for i in range(n)]
    outs = [torch.zeros((1, H), device=cuda) for _ in range(n)]
    st = pkg.Stack([layers[i % 2] for i in range(n)], xs, lgs, outs)
    for rep in range(2):
        st.run()
        torch.cuda.synchronize()
        assert pkg.moe_cache.device_error() == 0
        for i in range(n):
            assert torch.equal(outs[i], layers[i % 2].decode(xs[i], lgs[i])), (rep, i)


KT = (O.Q2_K, O.Q3_K, O.Q4_K, O.Q6_K)


@pytest.mark.parametrize("shape,pairs", [
    # every (gate/up, down) pair of the four K-quant types, one per layer
    ((1024, 512, 16, 4), [(a, b) for a in KT for b in KT]),
    # config-3 shapes, layer types as its seeded draws give them
    ((3072, 768, 64, 8), [(O.Q3_K, O.Q6_K), (O.Q2_K, O.Q2_K), (O.Q6_K, O.Q3_K), (O.Q4_K, O.Q2_K),
                          (O.Q2_K, O.Q4_K), (O.Q6_K, O.Q6_K)]),
], ids=["all-pairs", "config3-shapes"])
def test_mixed_type_stack_equals_layer_by_layer(pkg, cuda, shape, pairs):
    """Layers of different types in one launch (the mixed-type kernel): each
    layer's output and residual equal moe_b200_layer_decode bit for bit."""
    H, F, E, k = shape
    n = len(pairs)
    layers = [pkg.MoELayer(H, F, E, k, {"gate": a, "up": a, "down": b}, shared=True, seed=90 + l)
              for l, (a, b) in enumerate(pairs)]
    xs = [torch.zeros((1, H), device=cuda) for _ in range(n + 1)]
    xs[0].copy_(torch.from_numpy(activations((1, H), seed=5)))
    lgs = [torch.from_numpy(zipf_logits(1, E, seed=30 + l)).to(cuda) for l in range(n)]
    outs = [torch.zeros((1, H), device=cuda) for _ in range(n)]
    st = pkg.Stack(layers, xs[:n], lgs, outs, x_nexts=xs[1:])
    for rep in range(2):
        st.run()
        torch.cuda.synchronize()
        assert pkg.moe_cache.device_error() == 0
        x = xs[0].clone()
        for l in range(n):
            ref = layers[l].decode(x, lgs[l])
            assert torch.equal(outs[l], ref), (rep, l, pairs[l])
            x = x + ref
            assert torch.equal(xs[l + 1], x), (rep, l)


@pytest.mark.parametrize("pairs", [[(O.Q2_K, O.Q2_K)] * 4, [(O.Q3_K, O.Q6_K), (O.Q2_K, O.Q2_K), (O.Q6_K, O.Q4_K),
                                                           (O.Q4_K, O.Q3_K)]], ids=["q2k", "mixed"])
def test_stack_512_experts_equals_layer_by_layer(pkg, cuda, pairs):
    """Full-width layers (H=3072, F=768, 512 experts, top-8, shared expert):
    the stack equals the layer decode bit for bit."""
    H, F, E, k = 3072, 768, 512, 8
    n = len(pairs)
    layers = [pkg.MoELayer(H, F, E, k, {"gate": a, "up": a, "down": b}, shared=True, seed=120 + l)
              for l, (a, b) in enumerate(pairs)]
    xs = [torch.zeros((1, H), device=cuda) for _ in range(n + 1)]
    xs[0].copy_(torch.from_numpy(activations((1, H), seed=6)))
    lgs = [torch.from_numpy(zipf_logits(1, E, seed=40 + l)).to(cuda) for l in range(n)]
    outs = [torch.zeros((1, H), device=cuda) for _ in range(n)]
    st = pkg.Stack(layers, xs[:n], lgs, outs, x_nexts=xs[1:])
    st.run()
    torch.cuda.synchronize()
    assert pkg.moe_cache.device_error() == 0
    x = xs[0].clone()
    diffs = []
    for l in range(n):
        ref = layers[l].decode(x, lgs[l])
        diffs.append((l, float((outs[l] - ref).abs().max()), float(ref.abs().max())))
        x = x + ref
    assert all(d == 0.0 for _, d, _ in diffs), diffs


def test_stack_without_shared_expert(pkg, cuda):
    """Config-1 layers (H=2048, F=512, 64 experts, Q4_0, no shared expert) as
    a residual chain: equal to the layer decode bit for bit."""
    H, F, E, k, t = 2048, 512, 64, 8, O.Q4_0
    n = 5
    layers = [pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=False, seed=140 + l) for l in range(n)]
    xs = [torch.zeros((1, H), device=cuda) for _ in range(n + 1)]
    xs[0].copy_(torch.from_numpy(activations((1, H), seed=8)))
    lgs = [torch.from_numpy(activations((1, E), seed=60 + l)).to(cuda) for l in range(n)]
    outs = [torch.zeros((1, H), device=cuda) for _ in range(n)]
    st = pkg.Stack(layers, xs[:n], lgs, outs, x_nexts=xs[1:])
    st.run()
    torch.cuda.synchronize()
    assert pkg.moe_cache.device_error() == 0
    x = xs[0].clone()
    for l in range(n):
        ref = layers[l].decode(x, lgs[l])
        assert torch.equal(outs[l], ref), l
        x = x + ref
        assert torch.equal(xs[l + 1], x), l
