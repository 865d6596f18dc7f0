"""Expert-parallel decode (a6000-custom-kernels_b200/ep.py,
moe_b200_ep_layer_decode): each rank's share, summed over ranks, equals the
single-GPU layer. The ranks are emulated one after another on one GPU (the sum
is what the all-reduce computes); with two or more GPUs a real NCCL run is
checked too."""
import os

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


def _ep(pkg):
    from importlib import import_module
    return import_module("a6000-custom-kernels_b200.ep")


@pytest.mark.parametrize("world,n_tok,types", [(2, 1, (O.Q2_K, O.Q2_K, O.Q2_K)), (4, 3, (O.Q4_K, O.Q4_K, O.Q6_K)),
                                               (8, 8, (O.Q3_K, O.Q3_K, O.Q2_K)), (3, 2, (O.Q4_0, O.Q4_0, O.Q8_0))])
def test_rank_shares_sum_to_the_layer(pkg, cuda, world, n_tok, types):
    ep = _ep(pkg)
    H, F, E, k = 1024, 512, 64, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=True, seed=9)
    x = torch.from_numpy(activations((n_tok, H), seed=3)).to(cuda)
    lg = torch.from_numpy(zipf_logits(n_tok, E, seed=4)).to(cuda)
    pkg.moe_cache.set_layer_fused(False)      # the four-launch path: same pick-order combine per rank
    ref = full.decode(x, lg).cpu().numpy()
    ids_ref = full.routing_of(n_tok)[0].cpu().numpy()
    pkg.moe_cache.set_layer_fused(True)
    total = np.zeros_like(ref)
    for r in range(world):
        part = ep.EPMoELayer(full, r, world).partial(x, lg).cpu().numpy()
        total += part
    assert pkg.moe_cache.device_error() == 0
    err = np.abs(total - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
    # every rank routed the same picks
    lo, hi = ep.expert_range(E, 1 % world, world)
    assert ids_ref.min() >= 0 and ids_ref.max() < E and hi > lo


def _nccl_worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    pkg.moe_cache.configure(enabled=True)
    H, F, E, k = 1024, 512, 64, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": 10, "up": 10, "down": 10}, shared=True, seed=9, device=f"cuda:{rank}")
    x = torch.from_numpy(activations((2, H), seed=3)).cuda()
    lg = torch.from_numpy(zipf_logits(2, E, seed=4)).cuda()
    pkg.moe_cache.set_layer_fused(False)
    ref = full.decode(x, lg)
    out = ep.EPMoELayer(full, rank, world).decode(x, lg)
    torch.cuda.synchronize()
    err = float((out - ref).abs().max() / ref.abs().max())
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, err))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_all_reduce_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert all(e < 1e-5 for e in res.values()), res


@pytest.mark.parametrize("world,types", [(2, (O.Q2_K, O.Q2_K, O.Q2_K)), (3, (O.Q4_K, O.Q4_K, O.Q6_K)),
                                         (5, (O.Q3_K, O.Q3_K, O.Q2_K))])
def test_prefill_emulated_ranks_equal_layer_prefill(pkg, cuda, world, types):
    """Expert-parallel prefill (each rank its own prompt, experts spread over
    the ranks, dispatch / combine by all-to-all) emulated on one GPU: every
    rank's output equals the single-GPU layer prefill of its prompt bit for
    bit (each (row, token) result is independent of which tokens share its
    tile)."""
    ep = _ep(pkg)
    H, F, E, k = 1024, 512, 40, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=True, seed=21)
    ranks = [ep.EPMoELayer(full, r, world) for r in range(world)]
    xs = [torch.from_numpy(activations((24 + 5 * r, H), seed=30 + r)).to(cuda) for r in range(world)]
    lgs = [torch.from_numpy(zipf_logits(24 + 5 * r, E, seed=40 + r)).to(cuda) for r in range(world)]
    outs = ep.prefill_emulated(ranks, xs, lgs)
    assert pkg.moe_cache.device_error() == 0
    for r in range(world):
        ref = full.prefill(xs[r], lgs[r]).cpu().numpy()
        np.testing.assert_array_equal(outs[r].cpu().numpy(), ref)


def _nccl_prefill_worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    pkg.moe_cache.configure(enabled=True)
    H, F, E, k = 1024, 512, 64, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": 10, "up": 10, "down": 10}, shared=True, seed=9, device=f"cuda:{rank}")
    x = torch.from_numpy(activations((40 + 3 * rank, H), seed=50 + rank)).cuda()
    lg = torch.from_numpy(zipf_logits(40 + 3 * rank, E, seed=60 + rank)).cuda()
    ref = full.prefill(x, lg)
    out = ep.EPMoELayer(full, rank, world).prefill(x, lg)
    torch.cuda.synchronize()
    err = float((out - ref).abs().max())
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, err))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_prefill_all_to_all_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_nccl_prefill_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert all(e == 0.0 for e in res.values()), res


@pytest.mark.parametrize("world,types", [(2, (O.Q2_K, O.Q2_K, O.Q2_K)), (3, (O.Q4_K, O.Q4_K, O.Q6_K)),
                                         (4, (O.Q3_K, O.Q3_K, O.Q2_K))])
def test_prefill_peer_exchange_emulated(pkg, cuda, world, types):
    """The peer-memory exchange (dispatch straight into the owners' regions,
    empty slots marked -1, the owners' experts on the received rows with the
    quantization and the GLU inside the gathers, outputs written back) with
    the ranks emulated on one GPU: every rank's output equals the single-GPU
    layer prefill of its prompt bit for bit, over two layer calls (the
    arrival counters and regions are reused)."""
    ep = _ep(pkg)
    H, F, E, k = 1024, 512, 40, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=True, seed=23)
    ranks = [ep.EPMoELayer(full, r, world) for r in range(world)]
    n = [24 + 5 * r for r in range(world)]
    cap = max(n) * k
    exs = [ep.PeerExchange(H, cap, r, world) for r in range(world)]
    for ex in exs:
        ex.connect(peers=exs)
    try:
        for call in range(2):
            xs = [torch.from_numpy(activations((n[r], H), seed=70 + 10 * call + r)).to(cuda) for r in range(world)]
            lgs = [torch.from_numpy(zipf_logits(n[r], E, seed=90 + 10 * call + r)).to(cuda) for r in range(world)]
            outs = ep.prefill_p2p_emulated(ranks, exs, xs, lgs)
            assert pkg.moe_cache.device_error() == 0
            for r in range(world):
                np.testing.assert_array_equal(outs[r].cpu().numpy(), full.prefill(xs[r], lgs[r]).cpu().numpy())
    finally:
        torch.cuda.synchronize()
        for ex in exs:
            ex.close()


def _p2p_worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    pkg.moe_cache.configure(enabled=True)
    H, F, E, k = 1024, 512, 64, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": 10, "up": 10, "down": 12}, shared=True, seed=9, device=f"cuda:{rank}")
    L = ep.EPMoELayer(full, rank, world)
    n = 40 + 3 * rank
    ex = ep.PeerExchange(H, 43 * k, rank, world).connect()
    errs = []
    for call in range(3):
        x = torch.from_numpy(activations((n, H), seed=50 + 7 * call + rank)).cuda()
        lg = torch.from_numpy(zipf_logits(n, E, seed=60 + 7 * call + rank)).cuda()
        ref = full.prefill(x, lg)
        out = ep.prefill_p2p(L, ex, x, lg)
        torch.cuda.synchronize()
        errs.append(float((out - ref).abs().max()))
    code = pkg.moe_cache.device_error()
    dist.barrier()
    ex.close()
    dist.destroy_process_group()
    q.put((rank, max(errs), code))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_prefill_peer_exchange_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29650 + os.getpid() % 1000
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    res = [q.get(timeout=5) for _ in range(2)]
    assert all(p.exitcode == 0 for p in procs)
    for rank, err, code in res:
        assert code == 0 and err == 0.0, (rank, err, code)


def _fused_ep_reference(pkg, full, x, lg):
    pkg.moe_cache.set_layer_fused(False)          # the four-launch path: the same arithmetic, pick-order combine
    ref = full.decode(x, lg).clone()
    pkg.moe_cache.set_layer_fused(True)
    return ref


@pytest.mark.parametrize("types", [(O.Q2_K, O.Q2_K, O.Q2_K), (O.Q4_K, O.Q4_K, O.Q6_K)])
def test_fused_ep_decode_one_gpu(pkg, cuda, types):
    """The fused expert-parallel decode with world = 1 (the GPU exchanges with
    itself: gather slot, arrival word, returned rows and row counters all take
    the real path) equals the single-GPU layer bit for bit, over calls that
    alternate the gather parity, eagerly and replayed from a CUDA graph."""
    ep = _ep(pkg)
    H, F, E, k = 3072, 768, 512, 8
    full = pkg.MoELayer(H, F, E, k, {"gate": types[0], "up": types[1], "down": types[2]}, shared=True, seed=31)
    L = ep.EPMoELayer(full, 0, 1)
    ex = ep.DecodeExchange(H, E, k, 0, 1).connect()
    try:
        xs = [torch.from_numpy(activations((1, H), seed=80 + i)).to(cuda) for i in range(5)]
        lgs = [torch.from_numpy(zipf_logits(1, E, seed=90 + i)).to(cuda) for i in range(5)]
        refs = [_fused_ep_reference(pkg, full, xs[i], lgs[i]) for i in range(5)]
        for i in range(5):
            out = L.decode_p2p(ex, xs[i], lgs[i])
            assert pkg.moe_cache.device_error() == 0
            assert torch.equal(out, refs[i]), i
        s = torch.cuda.Stream()
        outs = torch.zeros((5, 1, H), device=cuda)
        with torch.cuda.stream(s):
            L.decode_p2p(ex, xs[0], lgs[0], outs[0], stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(5):
                L.decode_p2p(ex, xs[i], lgs[i], outs[i], stream=s)
        for _ in range(3):
            outs.zero_()
            g.replay()
            torch.cuda.synchronize()
            for i in range(5):
                assert torch.equal(outs[i], refs[i]), i
        del g
        assert pkg.moe_cache.device_error() == 0
    finally:
        torch.cuda.synchronize()
        ex.close()


def _fused_ep_worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    pkg.moe_cache.configure(enabled=True)
    pkg.moe_cache.set_wait_limits(0, 5_000_000_000)
    H, F, E, k = 3072, 768, 512, 8
    layers = [pkg.MoELayer(H, F, E, k, {"gate": 10, "up": 10, "down": t}, shared=True, seed=40 + t,
                           device=f"cuda:{rank}") for t in (10, 12)]
    shards = [ep.EPMoELayer(full, rank, world) for full in layers]
    ex = ep.DecodeExchange(H, E, k, rank, world).connect()
    worst, codes = 0.0, []
    for call in range(6):
        full, L = layers[call % 2], shards[call % 2]
        x = torch.from_numpy(activations((1, H), seed=100 + 10 * call + rank)).cuda()
        lg = torch.from_numpy(zipf_logits(1, E, seed=200 + 10 * call + rank)).cuda()
        ref = _fused_ep_reference(pkg, full, x, lg)
        out = L.decode_p2p(ex, x, lg)
        torch.cuda.synchronize()
        worst = max(worst, float((out - ref).abs().max()))
        codes.append(pkg.moe_cache.device_error())
    dist.barrier()
    ex.close()
    dist.destroy_process_group()
    q.put((rank, worst, max(codes)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_ep_decode_two_gpus():
    """Two GPUs, one token each, 512 experts split 256/256, the exchange inside
    the layer kernel over NVLink peer memory: each GPU's output equals the
    single-GPU layer of its token bit for bit, over six calls of two layers."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29750 + os.getpid() % 1000
    procs = [ctx.Process(target=_fused_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = [q.get(timeout=5) for _ in range(2)]
    assert all(p.exitcode == 0 for p in procs)
    for rank, err, code in res:
        assert code == 0 and err == 0.0, (rank, err, code)
