"""The cache-policy model (oracle/cache_model.py) against the rules of the
reference's registry and step (kernels/moe-cache.cu:525-775)."""
from cache_model import MAX_PROMOTIONS, CacheModel, parse_seed


def test_slot_sizing_budget_and_cap():
    m = CacheModel(slots=10, budget_bytes=25 * 100)
    a = m.register("a", "a", n_experts=16, expert_bytes=100)
    b = m.register("b", "b", n_experts=16, expert_bytes=100)
    c = m.register("c", "c", n_experts=4, expert_bytes=100)
    assert (a.n_slots, b.n_slots, c.n_slots) == (10, 10, 4 if 5 >= 4 else 5)
    assert m.register("a", "a", 16, 100) is a


def test_seed_fills_slots_in_order_and_skips_invalid():
    seed = parse_seed("t 5,5,99,3,-1,7,1\nother 1,2\n")
    assert seed["t"] == [5, 5, 99, 3, -1, 7, 1]
    m = CacheModel(slots=3, budget_bytes=1 << 40, seed=seed)
    t = m.register("t", "t", 8, 10)
    assert t.expert_of == [5, 3, 7]
    assert t.slot_of[5] == 0 and t.slot_of[3] == 1 and t.slot_of[7] == 2 and t.slot_of[1] == -1


def test_admission_on_second_sighting():
    m = CacheModel(slots=4, budget_bytes=1 << 40)
    t = m.register("t", "t", 8, 10)
    m.launch(t, [2])
    assert m.step() == 0 and t.slot_of[2] == -1
    m.launch(t, [2])
    assert m.step() == 1 and t.slot_of[2] == 0
    m.launch(t, [2])                      # now a hit
    assert m.step() == 0 and m.hits == 1


def test_two_sightings_in_one_step_promote():
    m = CacheModel(slots=4, budget_bytes=1 << 40)
    t = m.register("t", "t", 8, 10)
    m.launch(t, [6, 6, 6])                # 3 tokens picked expert 6
    assert m.step() == 1 and t.slot_of[6] == 0
    assert m.admission[(t.id << 12) | 6] == 1   # the third sighting was counted after the reset


def test_lru_victim_lowest_stamp_then_lowest_slot():
    m = CacheModel(slots=2, budget_bytes=1 << 40)
    t = m.register("t", "t", 8, 10)
    for e in (0, 1):
        m.launch(t, [e, e]); m.step()
    assert t.expert_of == [0, 1]
    m.launch(t, [1]); m.step()            # expert 1 newer than expert 0
    m.launch(t, [5, 5]); m.step()
    assert t.expert_of == [5, 1] and t.slot_of[0] == -1


def test_promotion_cap():
    m = CacheModel(slots=100, budget_bytes=1 << 40)
    t = m.register("t", "t", 100, 10)
    m.launch(t, [e for e in range(60) for _ in range(2)])
    assert m.step() == MAX_PROMOTIONS
    assert sum(s >= 0 for s in t.slot_of) == MAX_PROMOTIONS
    assert all(t.slot_of[e] >= 0 for e in range(MAX_PROMOTIONS))   # sorted order: lowest ids first


def test_sorted_order_is_tensor_major():
    m = CacheModel(slots=2, budget_bytes=1 << 40)
    a = m.register("a", "a", 8, 10)
    b = m.register("b", "b", 8, 10)
    m.launch(b, [1, 1]); m.launch(a, [3, 3, 2, 2])
    m.step()
    assert a.expert_of == [2, 3] and b.expert_of == [1, -1]
