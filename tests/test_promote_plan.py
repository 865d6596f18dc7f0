"""The promotion pass runs on the GPU as a parallel plan (moe_promote.cu):
distinct keys with multiplicities, one attempt flag per key, promotion
indices by prefix sum, a cut at the 48th promotion, then slot choice per
tensor. This restates that plan in Python and checks, on random logs, that it
leaves exactly the state the sequential policy model (oracle/cache_model.py,
the reference's loop) leaves: same slots, same admission counts, same
promotion count -- including steps that hit the 48-promotion cap."""
import random

import pytest

from cache_model import MAX_PROMOTIONS, CacheModel


def parallel_plan(model, log):
    """One step the way promote_kernel decides it."""
    keys = sorted(log)
    runs = []
    for k in keys:
        if runs and runs[-1][0] == k:
            runs[-1][1] += 1
        else:
            runs.append([k, 1])
    model.clock += 1
    flags = []
    for key, m in runs:
        cid, e = key >> 12, key & 0xFFF
        ok = False
        if cid < len(model.tensors):
            t = model.tensors[cid]
            seen = model.admission.get(key, 0)
            ok = e < t.n_experts and seen + m >= 2 and t.n_slots > 0 and t.slot_of[e] < 0
        flags.append(ok)
    index, n = [], 0
    for f in flags:
        index.append(n)
        n += f
    cut = next((j for j, f in enumerate(flags) if f and index[j] == MAX_PROMOTIONS - 1), None)
    for j, (key, m) in enumerate(runs):
        if cut is not None and j > cut:
            continue
        cid, e = key >> 12, key & 0xFFF
        if cid >= len(model.tensors) or e >= model.tensors[cid].n_experts:
            continue
        model.admission[key] = 0 if j == cut else (model.admission.get(key, 0) + m) % 2
    promoted = [runs[j][0] for j, f in enumerate(flags) if f and index[j] < MAX_PROMOTIONS]
    for key in promoted:
        t = model.tensors[key >> 12]
        e = key & 0xFFF
        slot = _acquire(t)
        t.slot_of[e] = slot
        t.expert_of[slot] = e
    model.promotions += len(promoted)
    return len(promoted)


def _acquire(t):
    for s in range(t.n_slots):
        if t.expert_of[s] < 0:
            return s
    best, vs = 0xFFFFFFFF, -1
    for s in range(t.n_slots):
        stamp = t.stamps[t.expert_of[s]]
        if stamp < best:
            best, vs = stamp, s
    victim = t.expert_of[vs]
    t.slot_of[victim] = -1
    t.expert_of[vs] = -1
    return vs


def _state(m):
    adm = {k: v for k, v in m.admission.items() if v}
    return [(t.slot_of, t.expert_of) for t in m.tensors], adm, m.promotions


@pytest.mark.parametrize("seed", range(12))
def test_parallel_plan_equals_sequential_policy(seed):
    rng = random.Random(seed)
    n_tensors = rng.choice([1, 3, 18, 40])
    slots = rng.choice([0, 1, 3, 8])
    E = rng.choice([8, 64, 512])
    a, b = CacheModel(slots=slots), CacheModel(slots=slots)
    for tid in range(n_tensors):
        for m in (a, b):
            m.register(tid, f"t{tid}", E, 1024)
    for step in range(30):
        for m in (a, b):
            m.log = []
        hot = rng.randint(1, E)
        for tid in range(n_tensors):
            entries = [min(E - 1, int(rng.paretovariate(1.1)) - 1) if rng.random() < 0.7 else rng.randrange(hot)
                       for _ in range(rng.choice([1, 8, 64]))]
            for m in (a, b):
                m.launch(m.tensors[tid], entries)
        log = list(b.log)
        b.log = []
        pa = a.step()
        pb = parallel_plan(b, log)
        assert pa == pb, (step, pa, pb)
        assert _state(a) == _state(b), step
    assert a.promotions > 0 or slots == 0
