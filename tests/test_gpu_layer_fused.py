"""The one-kernel layer decodes -- moe_layer2_kernel (per-expert CTA groups,
mode 1, the default) and moe_layer_kernel (grid-wide exchange of h, mode 2)
-- against the four-launch path: every intermediate and the output bit for bit, in eager
mode, under CUDA-graph replay, and for host-tiered experts. Oracle parity of
the fused path itself is covered by test_gpu_layer.py and test_gpu_cache.py,
which run it by default."""
import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, zipf_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    pkg.moe_cache.set_layer_fused(True)
    yield
    pkg.moe_cache.set_layer_fused(True)
    pkg.moe_cache.reset()


def _run(pkg, layer, x, lg, fused):
    pkg.moe_cache.set_layer_fused(fused)
    assert layer.fused(x.shape[0]) == bool(fused)
    out = layer.decode(x, lg)
    torch.cuda.synchronize()
    assert pkg.moe_cache.device_error() == 0
    return [t.cpu().numpy().copy() for t in layer.intermediates(x.shape[0])] + [out.cpu().numpy()]


NAMES = ("ids", "w", "h", "hs", "y", "ys", "out")


@pytest.mark.parametrize("types,n_tok,shape", [
    ((O.Q2_K, O.Q2_K), 1, (3072, 768, 512, 8)),        # config 2
    ((O.Q2_K, O.Q2_K), 8, (3072, 768, 512, 8)),
    ((O.Q2_K, O.Q2_K), -8, (3072, 768, 512, 8)),       # 8 tokens, unskewed routing: 64 distinct experts
    ((O.Q3_K, O.Q6_K), 3, (1024, 512, 64, 8)),
    ((O.Q6_K, O.Q4_K), 2, (2048, 256, 40, 6)),
    ((O.Q4_K, O.Q2_K), 5, (512, 1024, 16, 4)),
    ((O.Q4_0, O.Q4_0), 1, (2048, 512, 64, 8)),          # config 1 shape
    ((O.Q8_0, O.Q8_0), 4, (1024, 512, 32, 8)),
    ((O.Q5_0, O.Q5_0), 2, (512, 256, 16, 2)),
    ((O.Q5_K, O.Q5_K), 7, (512, 512, 128, 8)),
])
@pytest.mark.parametrize("mode", [1, 2])
def test_fused_matches_four_launches(pkg, cuda, types, n_tok, shape, mode):
    """n_tok < 0: |n_tok| tokens with N(0, 1) logits (no Zipf skew)."""
    H, F, E, k = shape
    ta, tb = types
    uniform = n_tok < 0
    n_tok = abs(n_tok)
    layer = pkg.MoELayer(H, F, E, k, {"gate": ta, "up": ta, "down": tb}, shared=True, seed=sum(types) + n_tok)
    x = torch.from_numpy(activations((n_tok, H), seed=11)).to(cuda)
    lg_np = activations((n_tok, E), seed=12) if uniform else zipf_logits(n_tok, E, seed=12)
    lg = torch.from_numpy(lg_np).to(cuda)
    a = _run(pkg, layer, x, lg, mode)
    b = _run(pkg, layer, x, lg, False)
    for name, u, v in zip(NAMES, a, b):
        np.testing.assert_array_equal(u, v, err_msg=name)
    # a second launch on the same workspace (epoch and row counters carried over)
    c = _run(pkg, layer, x, lg, mode)
    np.testing.assert_array_equal(c[-1], b[-1], err_msg="out, second launch")


def test_fused_without_shared_expert(pkg, cuda):
    H, F, E, k, n_tok = 1024, 512, 32, 8, 2
    layer = pkg.MoELayer(H, F, E, k, {"gate": O.Q2_K, "up": O.Q2_K, "down": O.Q2_K}, shared=False, seed=5)
    x = torch.from_numpy(activations((n_tok, H), seed=13)).to(cuda)
    lg = torch.from_numpy(zipf_logits(n_tok, E, seed=14)).to(cuda)
    a = _run(pkg, layer, x, lg, True)
    b = _run(pkg, layer, x, lg, False)
    for name, u, v in zip(NAMES, a, b):
        if name in ("hs", "ys"):
            continue
        np.testing.assert_array_equal(u, v, err_msg=name)


def test_fused_under_graph_replay(pkg, cuda):
    """Captured once, replayed many times: the grid barrier words return to
    zero after every launch, so every replay gives the eager result."""
    H, F, E, k = 3072, 768, 512, 8
    layers = [pkg.MoELayer(H, F, E, k, {"gate": O.Q2_K, "up": O.Q2_K, "down": O.Q2_K}, shared=True, seed=s)
              for s in range(2)]
    P = 4
    xs = torch.from_numpy(activations((P, 1, H), seed=21)).to(cuda)
    lgs = torch.from_numpy(zipf_logits(P, E, seed=22)).to(cuda).view(P, 1, E)
    outs = torch.zeros((P, 1, H), device=cuda)
    s = torch.cuda.Stream()
    ref = []
    with torch.cuda.stream(s):
        for i in range(P):
            ref.append(layers[i % 2].decode(xs[i], lgs[i], stream=s).clone())
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(P):
            layers[i % 2].decode(xs[i], lgs[i], outs[i], stream=s)
    for _ in range(25):
        outs.zero_()
        g.replay()
        torch.cuda.synchronize()
        for i in range(P):
            assert torch.equal(outs[i], ref[i])
    assert pkg.moe_cache.device_error() == 0
    del g


def test_fused_query(pkg, cuda):
    H, F, E, k = 512, 256, 16, 4
    mixed = pkg.MoELayer(H, F, E, k, {"gate": O.Q4_K, "up": O.Q4_K, "down": O.Q5_K}, shared=True, seed=1)
    assert not mixed.fused(1)                   # no fused kernel for this type pair
    same = pkg.MoELayer(H, F, E, k, {"gate": O.Q4_K, "up": O.Q4_K, "down": O.Q4_K}, shared=True, seed=1)
    assert same.fused(1) and same.fused(8)
    pkg.moe_cache.set_layer_fused(False)
    assert not same.fused(1)


def test_one_workspace_for_many_layers_and_batch_sizes(pkg, cuda):
    """One caller-owned workspace (zero-filled once) serves two layers and
    several batch sizes in turn: the launch epoch at its start keeps every
    launch's exchanged data apart."""
    import ctypes
    from importlib import import_module
    lib = import_module("a6000-custom-kernels_b200._lib").lib()
    H, F, E, k = 1024, 512, 64, 8
    layers = [pkg.MoELayer(H, F, E, k, {"gate": O.Q2_K, "up": O.Q2_K, "down": O.Q2_K}, shared=True, seed=s)
              for s in (31, 32)]
    nbytes = max(lib.moe_b200_layer_workspace_size(ctypes.byref(L.desc), n) for L in layers for n in (1, 2, 3))
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    for i, n in enumerate((1, 2, 1, 3, 3, 2, 1, 1)):
        L = layers[i % 2]
        x = torch.from_numpy(activations((n, H), seed=40 + i)).to(cuda)
        lg = torch.from_numpy(zipf_logits(n, E, seed=50 + i)).to(cuda)
        out = torch.empty((n, H), device=cuda)
        rc = lib.moe_b200_layer_decode(ctypes.byref(L.desc), x.data_ptr(), lg.data_ptr(), out.data_ptr(), n,
                                       ws.data_ptr(), nbytes, None)
        assert rc == 0
        pkg.moe_cache.set_layer_fused(False)
        ref = L.decode(x, lg)
        pkg.moe_cache.set_layer_fused(True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), i
    assert pkg.moe_cache.device_error() == 0
