"""Routing trace and seed-file builder (a6000-custom-kernels_b200/seed.py)
against fixtures made by running the reference's tools/make_seed.py on a
synthetic trace (tests/golden/seed/make_seed_fixture.py): the seed text is
identical, and the trace writer produces the fixture's bytes."""
import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "seed")


def _seed():
    return importlib.import_module("a6000-custom-kernels_b200.seed")


def test_seed_file_matches_reference_builder(tmp_path):
    out = tmp_path / "seed.txt"
    _seed().build_seed(os.path.join(GOLD, "trace.bin"), str(out))
    assert out.read_text() == open(os.path.join(GOLD, "seed_expected.txt")).read()


def test_trace_writer_bytes_match_fixture(tmp_path):
    sys.path.insert(0, GOLD)
    import make_seed_fixture as F
    path = tmp_path / "trace.bin"
    with _seed().TraceWriter(str(path)) as w:
        for name, ids, E in F.records():
            w.record(name, ids, E)
    assert path.read_bytes() == open(os.path.join(GOLD, "trace.bin"), "rb").read()


def test_trace_roundtrip_and_rules(tmp_path):
    import numpy as np
    S = _seed()
    path = tmp_path / "t.bin"
    with S.TraceWriter(str(path)) as w:
        w.record("a", [[3, 1]], 8)
        w.record("a", [[1, 5]], 8)
        w.record("b", [[2, 2]], 8)
        w.record("a", [[7, 7], [7, 7]], 8)     # two tokens: not a decode record
        w.record("a", [[9, 0]], 8)              # 9 is out of range
    recs = list(S.read_trace(str(path)))
    assert [r[0] for r in recs] == ["a", "a", "b", "a", "a"]
    assert np.array_equal(recs[3][2], [[7, 7], [7, 7]])
    # counts a: 1 x3, 3 x1, 5 x1, 0 x1 -> 1 first, then ties in first-seen order
    assert S.seed_order(str(path)) == {"a": [1, 3, 5, 0], "b": [2]}
