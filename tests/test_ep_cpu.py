"""Expert-parallel decomposition on CPU ranks (gloo, world size 2): every rank
routes all experts, computes the picks it holds with the CPU oracle, adds the
shared expert on rank 0, and an all-reduce of the shares gives the full
oracle layer. The partition is ep.expert_range, the share semantics are those
of moe_b200_ep_layer_decode (its picks in pick order, plus the shared
expert on rank 0)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _share(L, x, logits, lo, hi, with_shared):
    import oracle as O
    n_tok, k = x.shape[0], L["k"]
    ids, w = O.topk_softmax(logits, k)
    H, F = L["H"], L["F"]
    out = np.zeros((n_tok, H), np.float32)
    for t in range(n_tok):
        acc, anyp = np.float32(0), False
        first = True
        row = np.zeros(H, np.float32)
        for p in range(k):
            e = int(ids[t, p])
            if not (lo <= e < hi):
                continue
            one = np.array([[e]], np.int32)
            g = O.mul_mat_id(L["type_gate"], L["gate"], H, x[t:t + 1, None], one)
            u = O.mul_mat_id(L["type_up"], L["up"], H, x[t:t + 1, None], one)
            h = O.glu(O.GLU_SWIGLU, g, u)
            y = O.mul_mat_id(L["type_down"], L["down"], F, h, one)[0, 0]
            v = (y * w[t, p]).astype(np.float32)
            row = v if first else (row + v).astype(np.float32)
            first = False
        if with_shared:
            z = np.zeros((1, 1), np.int32)
            sg = O.mul_mat_id(L["type_gate"], L["shared_gate"][None], H, x[t:t + 1, None], z)
            su = O.mul_mat_id(L["type_up"], L["shared_up"][None], H, x[t:t + 1, None], z)
            ys = O.mul_mat_id(L["type_down"], L["shared_down"][None], F, O.glu(O.GLU_SWIGLU, sg, su), z)[0, 0]
            row = (row + ys).astype(np.float32)
        out[t] = row
    return out


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import importlib
    import torch
    import torch.distributed as dist
    import oracle as O
    from moe_data import activations, experts, zipf_logits
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    H, F, E, k, t = 256, 256, 16, 4, O.Q4_K
    L = dict(H=H, F=F, E=E, k=k, type_gate=t, type_up=t, type_down=t, gate=experts(t, E, F, H, 1),
             up=experts(t, E, F, H, 2), down=experts(t, E, H, F, 3), shared_type=t,
             shared_gate=experts(t, 1, F, H, 4)[0], shared_up=experts(t, 1, F, H, 5)[0],
             shared_down=experts(t, 1, H, F, 6)[0])
    x = activations((2, H), seed=7)
    logits = zipf_logits(2, E, seed=8)
    lo, hi = ep.expert_range(E, rank, world)
    share = torch.from_numpy(_share(L, x, logits, lo, hi, rank == 0))
    dist.all_reduce(share, op=dist.ReduceOp.SUM)
    ref = O.moe_layer(L, x, logits)[0]
    err = float(np.abs(share.numpy() - ref).max() / np.abs(ref).max())
    dist.destroy_process_group()
    q.put((rank, err, (lo, hi)))


def test_expert_ranges_cover_all_experts():
    sys.path.insert(0, ROOT)
    import importlib
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    for E in (16, 64, 512, 513):
        for world in (1, 2, 3, 4, 8):
            got = [ep.expert_range(E, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == E
            assert all(got[i][1] == got[i + 1][0] for i in range(world - 1))
            assert max(h - l for l, h in got) - min(h - l for l, h in got) <= 1


def test_gloo_two_ranks_sum_to_the_layer():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = [q.get(timeout=5) for _ in range(2)]
    assert all(p.exitcode == 0 for p in procs)
    for rank, err, rng in res:
        assert err < 1e-5, (rank, err)        # oracle layer vs shares: float summation order only


def _prefill_worker(rank, world, port, q):
    """dispatch / combine of the expert-parallel prefill on gloo: every entry's
    row reaches the rank owning its expert, and its output comes back to its
    (token, pick) slot. The stand-in expert is y = (global expert + 1) * x."""
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import importlib
    import torch
    import torch.distributed as dist
    ep = importlib.import_module("a6000-custom-kernels_b200.ep")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    E, k, H, n = 13, 3, 8, 7 + rank          # uneven expert slices, different token counts per rank
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn((n, H), generator=g)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(n)]).to(torch.int32)
    lo, hi = ep.expert_range(E, rank, world)
    seen = []

    def compute(rows, lids):
        seen.append(int(lids.numel()))
        if lids.numel():
            assert int(lids.min()) >= 0 and int(lids.max()) < hi - lo
        return rows * (lids.to(torch.float32) + lo + 1)[:, None]

    y = ep.exchange(x, ids, E, world, compute)
    ref = x[:, None, :] * (ids.to(torch.float32) + 1)[:, :, None]
    err = float((y - ref).abs().max())
    dist.destroy_process_group()
    q.put((rank, err, seen[0]))


def test_gloo_prefill_dispatch_combine():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 1000
    world = 3
    procs = [ctx.Process(target=_prefill_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = [q.get(timeout=5) for _ in range(world)]
    assert all(p.exitcode == 0 for p in procs)
    for rank, err, n_recv in res:
        assert err == 0.0, (rank, err)
    assert sum(r[2] for r in res) == sum(3 * (7 + r) for r in range(world))   # every entry computed once
