"""The tiered hot-expert cache on the GPU: experts in pinned host memory read
zero-copy through tagged table entries, a capped HBM pool, seeding, and the
promotion step. After every step the DEVICE pointer tables are read back and
compared bit-exactly with the policy model (oracle/cache_model.py), and the
layer outputs are checked against the CPU oracle while experts move."""
import numpy as np
import pytest
import torch

import oracle as O
from cache_model import CacheModel, parse_seed
from layer_check import check_layer
from moe_data import activations, experts, zipf_logits

pytestmark = pytest.mark.gpu
_KEEP_PINNED = []


def _layer_np(t, H, F, E, seed):
    return dict(H=H, F=F, E=E, type_gate=t, type_up=t, type_down=t,
                gate=experts(t, E, F, H, seed), up=experts(t, E, F, H, seed + 1), down=experts(t, E, H, F, seed + 2),
                shared_type=t, shared_gate=experts(t, 1, F, H, seed + 3)[0],
                shared_up=experts(t, 1, F, H, seed + 4)[0], shared_down=experts(t, 1, H, F, seed + 5)[0])


@pytest.mark.parametrize("n_tok,slots,fused", [(1, 5, True), (4, 3, True), (4, 3, False)])
def test_tiered_cache_matches_policy_model(pkg, cuda, tmp_path, n_tok, slots, fused):
    """fused: the one-kernel layer decode; else the four-launch path."""
    mc = pkg.moe_cache
    t, H, F, E, k = O.Q4_K, 512, 256, 16, 4
    L = _layer_np(t, H, F, E, seed=11)
    L["k"] = k
    seed_text = "blk.0.ffn_up_exps.weight 3,1,4,1,77\nblk.0.ffn_down_exps.weight 0,9\n"
    seed_file = tmp_path / "seed.txt"
    seed_file.write_text(seed_text)
    mc.configure(enabled=True, slots=slots, budget_gb=1.0, seed_path=str(seed_file))
    mc.set_layer_fused(fused)
    try:
        layer = pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, host=True,
                             weights={r: L[r] for r in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down")})
        assert all(mc.wants(layer.desc_t[r]) for r in ("gate", "up", "down"))
        assert layer.fused(n_tok) == fused
        model = CacheModel(slots=slots, budget_bytes=1 << 30, seed=parse_seed(seed_text))
        names = {r: f"blk.0.ffn_{r}_exps.weight" for r in ("gate", "up", "down")}
        eb = {r: layer.w[r][0].numel() for r in ("gate", "up", "down")}
        mt = {}
        for step in range(24):
            x = activations((n_tok, H), seed=100 + step)
            logits = zipf_logits(n_tok, E, seed=7) + 0.3 * activations((n_tok, E), seed=200 + step)
            out = layer.decode(torch.from_numpy(x).to(cuda), torch.from_numpy(logits).to(cuda))
            check_layer(layer, L, x, logits, out.cpu().numpy())
            ids = layer.routing_of(n_tok)[0].cpu().numpy()
            if step == 0:
                for r in ("up", "gate", "down"):          # registration order of the library
                    mt[r] = model.register(r, names[r], E, eb[r])
            entries = ids.reshape(-1).tolist()
            for r in ("up", "gate", "down"):
                model.launch(mt[r], entries)
            mc.step()
            model.step()
            for r in ("up", "gate", "down"):
                tbl, n_slots, tid = mc.table(layer.desc_t[r])
                assert n_slots == mt[r].n_slots and tid == mt[r].id
                assert tbl == mt[r].slot_of, (step, r)
        s = mc.stats()
        assert s["promotions"] == model.promotions and s["hits"] == model.hits
        assert s["promotions"] > 0 and s["evictions"] > 0
        assert mc.device_error() == 0
    finally:
        mc.set_layer_fused(True)
        mc.reset()


def test_pin_host_and_wants(pkg, cuda):
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    try:
        t, E, rows, K = O.Q8_0, 4, 8, 64
        arr = np.ascontiguousarray(experts(t, E, rows, K, seed=1))
        buf = torch.from_numpy(arr)                 # plain (unregistered) host memory
        d = mc.expert_tensor(buf, t, K, rows, name="plain")
        assert not mc.wants(d)
        assert mc.pin_host(d)
        assert mc.wants(d)
        dev = buf.to(cuda)
        assert mc.wants(mc.expert_tensor(dev, t, K, rows))
        assert not mc.pin_host(mc.expert_tensor(dev, t, K, rows))
        one = mc.expert_tensor(dev[:1].clone(), t, K, rows)
        assert not mc.wants(one)                     # ne[2] < 2
        view = mc.expert_tensor(dev, t, K, rows, flags=mc.TENSOR_VIEW)
        assert not mc.wants(view)
        _KEEP_PINNED.append(arr)          # registered pages stay valid until exit
    finally:
        mc.reset()


def test_device_resident_tables_are_direct(pkg, cuda):
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    try:
        t, H, F, E, k = O.Q2_K, 512, 256, 8, 2
        layer = pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=False, seed=1)
        layer.decode(torch.randn(1, H, device=cuda), torch.randn(1, E, device=cuda))
        mc.step()                                     # no host tensors: no sync, nothing to promote
        for r in ("gate", "up", "down"):
            tbl, n_slots, _ = mc.table(layer.desc_t[r])
            assert n_slots == 0 and tbl == [-2] * E
        assert mc.stats()["misses"] == 0
    finally:
        mc.reset()


def test_promotion_cap_and_many_tensors(pkg, cuda):
    """Six tiered layers at batch 8: every step logs several hundred misses
    with repeats over 18 tensors, more than 48 experts become candidates, so
    the per-step cap decides which keys are read; the device tables, slot
    maps and totals must still equal the policy model's after every step."""
    mc = pkg.moe_cache
    t, H, F, E, k, n_tok, slots, n_layers = O.Q2_K, 256, 256, 64, 8, 8, 6, 6
    mc.configure(enabled=True, slots=slots, budget_gb=4.0)
    try:
        layers, Ls = [], []
        for l in range(n_layers):
            L = _layer_np(t, H, F, E, seed=40 + 7 * l)
            L["k"] = k
            Ls.append(L)
            layers.append(pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, host=True,
                                       name=f"blk.{l}",
                                       weights={r: L[r] for r in ("gate", "up", "down", "shared_gate", "shared_up",
                                                                  "shared_down")}))
        model = CacheModel(slots=slots, budget_bytes=4 << 30)
        mt = {}
        capped = 0
        for step in range(10):
            for l, layer in enumerate(layers):
                x = activations((n_tok, H), seed=500 + 31 * step + l)
                logits = zipf_logits(n_tok, E, seed=60 + l) + 2.0 * activations((n_tok, E), seed=900 + 31 * step + l)
                out = layer.decode(torch.from_numpy(x).to(cuda), torch.from_numpy(logits).to(cuda))
                if step % 3 == 0:
                    check_layer(layer, Ls[l], x, logits, out.cpu().numpy())
                ids = layer.routing_of(n_tok)[0].cpu().numpy()
                if step == 0:
                    for r in ("up", "gate", "down"):
                        mt[(l, r)] = model.register((l, r), f"blk.{l}.ffn_{r}_exps.weight", E,
                                                    layer.w[r][0].numel())
                for r in ("up", "gate", "down"):
                    model.launch(mt[(l, r)], ids.reshape(-1).tolist())
            mc.step()
            capped += model.step() == 48
            for l, layer in enumerate(layers):
                for r in ("up", "gate", "down"):
                    tbl, n_slots, tid = mc.table(layer.desc_t[r])
                    assert tid == mt[(l, r)].id and n_slots == slots
                    assert tbl == mt[(l, r)].slot_of, (step, l, r)
        s = mc.stats()
        assert capped > 0, "no step reached the 48-promotion cap"
        assert s["promotions"] == model.promotions and s["hits"] == model.hits
        assert s["resident"] == sum(sum(1 for e in m.expert_of if e >= 0) for m in mt.values())
        assert mc.device_error() == 0
    finally:
        mc.reset()


def test_step_inside_a_cuda_graph(pkg, cuda):
    """The promotion step enqueues device work only, so decode + step can be
    captured in one CUDA graph; replaying it moves the cache exactly as the
    eager sequence does."""
    mc = pkg.moe_cache
    t, H, F, E, k = O.Q4_K, 256, 256, 32, 4
    L = _layer_np(t, H, F, E, seed=77)
    L["k"] = k
    w = {r: L[r] for r in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down")}
    x = torch.from_numpy(activations((2, H), seed=1)).to(cuda)
    lgs = [torch.from_numpy(zipf_logits(2, E, seed=3) + 1.5 * activations((2, E), seed=10 + i)).to(cuda)
           for i in range(4)]
    tables = []
    for graph in (False, True):
        mc.configure(enabled=True, slots=4, budget_gb=1.0)
        try:
            layer = pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, host=True, weights=w)
            stream = torch.cuda.Stream(cuda)
            out = torch.empty((2, H), device=cuda)
            with torch.cuda.stream(stream):
                layer.decode(x, lgs[0], out, stream=stream)   # registers the tensors (not capturable)
                mc.step(stream)
            stream.synchronize()

            def seq():
                for lg in lgs:
                    layer.decode(x, lg, out, stream=stream)
                    mc.step(stream)
            if graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    seq()
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                del g
            else:
                with torch.cuda.stream(stream):
                    for _ in range(3):
                        seq()
                stream.synchronize()
            tables.append([mc.table(layer.desc_t[r])[0] for r in ("gate", "up", "down")])
            s = mc.stats()
            tables[-1].append((s["promotions"], s["evictions"], s["hits"], s["misses"]))
            assert mc.device_error() == 0
        finally:
            mc.reset()
    assert tables[0] == tables[1]
    assert tables[0][-1][0] > 0
