"""Makes the seed-builder fixtures: a synthetic routing trace in the trace
hook's binary format (u32 namelen, u32 n_used, u32 n_tok, u32 n_exp, name,
i32 ids[n_tok * n_used]) and the seed file the reference's own
tools/make_seed.py builds from it. Run once in a container that has the
reference checkout:  python tests/golden/seed/make_seed_fixture.py <reference root>"""
import os
import struct
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def records():
    rng = np.random.default_rng(2024)
    names = [f"blk.{l}.ffn_{r}_exps.weight" for l in range(2) for r in ("gate", "up", "down")]
    out = []
    for step in range(60):
        for name in names:
            E, k = 64, 8
            perm = np.random.default_rng(sum(name.encode())).permutation(E)
            if step % 7 == 3:      # a prefill record (several tokens): not a decode pick
                n_tok = 5
            else:
                n_tok = 1
            ids = []
            for _ in range(n_tok):
                w = np.exp(-1.1 * np.log(perm + 1.0) + rng.normal(0, 1, E))
                ids.append(np.argsort(-w, kind="stable")[:k])
            ids = np.array(ids, dtype=np.int32)
            if step == 11:         # out-of-range ids are skipped by the builder
                ids[0, 0] = -1
                ids[0, 1] = E + 3
            out.append((name, ids, E))
    out.append(("blk.9.ffn_gate_exps.weight", np.array([[0]], np.int32), 1))   # n_exp < 2: skipped
    return out


def write_trace(path):
    with open(path, "wb") as f:
        for name, ids, E in records():
            nm = name.encode()
            f.write(struct.pack("<IIII", len(nm), ids.shape[1], ids.shape[0], E) + nm + ids.astype("<i4").tobytes())


if __name__ == "__main__":
    ref = sys.argv[1]
    trace = os.path.join(HERE, "trace.bin")
    write_trace(trace)
    subprocess.check_call([sys.executable, os.path.join(ref, "tools", "make_seed.py"), trace,
                           os.path.join(HERE, "seed_expected.txt")])
