"""Routing traces and hot-expert seed files.

The cache seeds each expert tensor's pool from a text file of lines
"tensorname id1,id2,..." (experts by decreasing decode-pick frequency; the
library reads it at configure time, GGML_CUDA_MOE_CACHE_SEED). This module
writes the routing trace such a file is made from and builds the file:

* trace format (the reference's trace hook, patches/trace-hook/ggml-cpu.c,
  read by tools/make_seed.py:27-37), per MUL_MAT_ID call:
  u32 namelen, u32 n_used, u32 n_tok, u32 n_exp, char name[namelen],
  i32 ids[n_tok * n_used] (token-major);
* seed rule (tools/make_seed.py:33-49): only decode records (n_tok == 1,
  n_exp >= 2), ids outside [0, n_exp) ignored; per tensor, experts ordered by
  pick count, descending, ties in order of first appearance; tensors in
  order of first appearance.
"""
import struct

import numpy as np


class TraceWriter:
    """Appends MUL_MAT_ID routing records to a trace file."""

    def __init__(self, path):
        self.f = open(path, "ab")

    def record(self, name, ids, n_experts):
        """ids: int [n_tok][n_used] (numpy, torch or nested lists)."""
        ids = np.asarray(ids.cpu() if hasattr(ids, "cpu") else ids, dtype=np.int32)
        if ids.ndim == 1:
            ids = ids[None]
        n_tok, n_used = ids.shape
        nm = name.encode()
        self.f.write(struct.pack("<IIII", len(nm), n_used, n_tok, n_experts) + nm)
        self.f.write(np.ascontiguousarray(ids, dtype="<i4").tobytes())

    def close(self):
        self.f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
        return False


def read_trace(path):
    """Yields (name, n_exp, ids [n_tok][n_used]) per record."""
    with open(path, "rb") as f:
        while True:
            hdr = f.read(16)
            if len(hdr) < 16:
                return
            namelen, n_used, n_tok, n_exp = struct.unpack("<IIII", hdr)
            name = f.read(namelen).decode("utf-8", "replace")
            ids = np.frombuffer(f.read(4 * n_used * n_tok), dtype="<i4").reshape(n_tok, n_used)
            yield name, n_exp, ids


def seed_order(trace_path):
    """{tensorname: [experts by decreasing decode-pick count]} in first-seen order."""
    order = {}          # name -> (counts dict, first-seen order of experts)
    for name, n_exp, ids in read_trace(trace_path):
        if ids.shape[0] != 1 or n_exp < 2:
            continue                                      # decode records only
        counts, seen = order.setdefault(name, ({}, []))
        for e in ids.reshape(-1).tolist():
            if 0 <= e < n_exp:
                if e not in counts:
                    counts[e] = 0
                    seen.append(e)
                counts[e] += 1
    out = {}
    for name, (counts, seen) in order.items():
        rank = {e: i for i, e in enumerate(seen)}
        out[name] = sorted(seen, key=lambda e: (-counts[e], rank[e]))
    return out


def build_seed(trace_path, out_path):
    """Writes the seed file for a trace; returns {tensorname: expert order}."""
    order = seed_order(trace_path)
    with open(out_path, "w") as f:
        for name, experts in order.items():
            f.write(name + " " + ",".join(str(e) for e in experts) + "\n")
    return order
