"""Generate the golden block-format fixtures in this folder.

The reference project ships no tests or golden vectors, and llama.cpp (the
third-party code that owns the block formats and quantizers, pinned by the
reference at llama.cpp commit 11fe0215, scripts/build.sh:14-20) is not present.
gguf-py 0.19.0 (llama.cpp's own Python package, installed in this image) is an
independent implementation of the same formats, so it generates the fixtures:

  dequant_<TYPE>.npz : random valid blocks -> gguf.quants.dequantize output
                       (all eight weight formats of the path)
  quant_<TYPE>.npz   : N(0, 0.02) rows -> gguf.quants.quantize output
                       (Q4_0, Q5_0, Q8_0: the formats gguf-py can quantize)

Run from the repository root: python tests/golden/make_golden.py
The fixtures are committed; tests read them and never import gguf.
"""
import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, ggml type id, block elems, block bytes, byte offsets of f16 scale fields)
TYPES = [
    ("Q4_0", T.Q4_0, 32, 18, [0]),
    ("Q5_0", T.Q5_0, 32, 22, [0]),
    ("Q8_0", T.Q8_0, 32, 34, [0]),
    ("Q2_K", T.Q2_K, 256, 84, [80, 82]),
    ("Q3_K", T.Q3_K, 256, 110, [108]),
    ("Q4_K", T.Q4_K, 256, 144, [0, 2]),
    ("Q5_K", T.Q5_K, 256, 176, [0, 2]),
    ("Q6_K", T.Q6_K, 256, 210, [208]),
]


def main():
    rng = np.random.default_rng(20261201)
    for name, gt, blck, tsize, half_offs in TYPES:
        nb = 24
        blocks = rng.integers(0, 256, size=(nb, tsize), dtype=np.uint8)
        for off in half_offs:
            h = rng.uniform(-0.05, 0.05, size=nb).astype(np.float16)
            blocks[:, off:off + 2] = h.view(np.uint8).reshape(nb, 2)
        deq = quants.dequantize(blocks.reshape(-1), gt).reshape(-1).astype(np.float32)
        np.savez_compressed(os.path.join(HERE, f"dequant_{name}.npz"), ggml_type=int(gt), blocks=blocks,
                            values=deq)
        if name in ("Q4_0", "Q5_0", "Q8_0"):
            x = rng.normal(0.0, 0.02, size=(8, 512)).astype(np.float32)
            x[0, :32] = 0.0                      # an all-zero block
            x[1, 5] = -x[1, 5:37].__abs__().max() * 1.5   # a negative extreme
            q = quants.quantize(x, gt)
            np.savez_compressed(os.path.join(HERE, f"quant_{name}.npz"), ggml_type=int(gt), x=x,
                                blocks=np.asarray(q, dtype=np.uint8))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
