"""Seeded synthetic inputs for the parity tests (shapes and distributions of
the benchmark configs: weights ~ N(0, 0.02) quantized, activations ~ N(0, 1),
router logits ~ N(0, 1) or Zipf(1.1)-skewed)."""
import numpy as np

import oracle as O


def experts(t, E, rows, K, seed, sigma=0.02):
    """uint8 [E][rows][row_bytes] of N(0, sigma) weights quantized by the oracle."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, sigma, size=(E * rows, K)).astype(np.float32)
    return O.quantize(t, x).reshape(E, rows, O.row_size(t, K))


def activations(shape, seed):
    return np.random.default_rng(seed).normal(0.0, 1.0, size=shape).astype(np.float32)


def zipf_logits(n_tok, E, seed, alpha=1.1):
    """log Zipf_alpha(rank pi(e)) + N(0, 1), pi a seeded permutation."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    base = -alpha * np.log(perm + 1.0)
    return (base[None, :] + rng.normal(0.0, 1.0, size=(n_tok, E))).astype(np.float32)


def distinct_ids(n_tok, n_used, E, seed):
    rng = np.random.default_rng(seed)
    return np.stack([rng.choice(E, size=n_used, replace=False) for _ in range(n_tok)]).astype(np.int32)


def rel_err(got, ref):
    """max |got - ref| / max |ref| per output vector (last axis), worst case."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    num = np.abs(got - ref).max(axis=-1)
    den = np.maximum(np.abs(ref).max(axis=-1), 1e-30)
    return float((num / den).max())
