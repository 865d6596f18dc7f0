"""The oracle's block formats and quantizers against the golden fixtures made
from gguf-py (tests/golden/make_golden.py)."""
import glob
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAME_TO_TYPE = {"Q4_0": O.Q4_0, "Q5_0": O.Q5_0, "Q8_0": O.Q8_0, "Q2_K": O.Q2_K, "Q3_K": O.Q3_K,
                "Q4_K": O.Q4_K, "Q5_K": O.Q5_K, "Q6_K": O.Q6_K}


@pytest.mark.parametrize("name", sorted(NAME_TO_TYPE))
def test_dequant_matches_gguf(name):
    f = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    t = NAME_TO_TYPE[name]
    assert int(f["ggml_type"]) == t
    blocks = f["blocks"]
    n = blocks.shape[0] * O.BLCK[t]
    got = O.dequantize(t, blocks, n).reshape(-1)
    np.testing.assert_array_equal(got, f["values"])


@pytest.mark.parametrize("name", ["Q4_0", "Q5_0", "Q8_0"])
def test_quantize_matches_gguf(name):
    f = np.load(os.path.join(GOLDEN, f"quant_{name}.npz"))
    t = NAME_TO_TYPE[name]
    got = O.quantize(t, f["x"]).reshape(-1)
    np.testing.assert_array_equal(got, f["blocks"].reshape(-1))


def test_all_fixtures_present():
    assert len(glob.glob(os.path.join(GOLDEN, "dequant_*.npz"))) == 8
    assert len(glob.glob(os.path.join(GOLDEN, "quant_*.npz"))) == 3


def test_fp16_roundtrip_exhaustive():
    L = O.lib()
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([L.orc_fp16_to_fp32(int(v)) for v in h], dtype=np.float32)
    finite = np.isfinite(ref)
    np.testing.assert_array_equal(got[finite], ref[finite])
    assert np.isnan(got[~finite & np.isnan(ref)]).all()


def test_fp32_to_fp16_rne():
    L = O.lib()
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 2000),
                        [0.0, -0.0, 65504.0, 65520.0, 1e9, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26]]).astype(np.float32)
    ref = x.astype(np.float16).view(np.uint16)
    got = np.array([L.orc_fp32_to_fp16(float(v)) for v in x], dtype=np.uint16)
    np.testing.assert_array_equal(got, ref)
