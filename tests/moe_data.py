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


def act_quant_sigma(t, W, K, x, ids):
    """Standard deviation of (result with Q8_1 activations) - (result with
    llama.cpp's CPU activations: Q8_K per 256 for K-quants, Q8_0 per 32
    otherwise) for every output [n_tok][n_used][rows] of a MUL_MAT_ID with
    one input row per token (x f32 [n_tok][K]). Both sides dot the same
    weights w (dequantized rows) with x rounded to their own grid; modelled
    as independent errors:
      * element rounding, uniform in +-d/2 with d the block's step
        (amax / 127): variance w_i^2 (d1_i^2 + dc_i^2) / 12;
      * the f16 block scales of Q8_1 and Q8_0 (relative error uniform in
        +-2^-11): variance (sum over the block of w_i x_i)^2 * 2^-22 / 3.
    Q4_0 / Q5_0 with Q8_1 activations (llama.cpp's CUDA dot) compute
    d_w (d_a sum(q_w q_a) - offset s), s the f16 sum of the unquantized x of
    the block: the Q8_1 side's rounding then meets the unsigned weights
    u_i = w_i + offset d_w (in both terms above), and s adds the variance
    (offset d_w)^2 (sum over the block of x_i)^2 2^-22 / 3.
    No test assumes more than this model."""
    import oracle as O
    x = np.asarray(x, dtype=np.float64)
    n_tok = x.shape[0]
    step = {}
    for name, blk in (("q8_1", 32), ("cpu", 256 if O.vec_dot_type(t) == O.Q8_K else 32)):
        xb = x.reshape(n_tok, K // blk, blk)
        d = np.abs(xb).max(axis=2) / 127.0
        step[name] = (np.repeat(d, blk, axis=1), blk)
    var_el = (step["q8_1"][0] ** 2 + step["cpu"][0] ** 2) / 12.0            # [n_tok][K]
    f16_cpu = O.vec_dot_type(t) == O.Q8_0
    off = {O.Q4_0: 8, O.Q5_0: 16}.get(t, 0)
    f16 = (2.0 ** -22) / 3.0
    out = np.zeros(ids.shape + (W.shape[1],))
    for ti in range(n_tok):
        for p in range(ids.shape[1]):
            w = O.dequantize(t, W[ids[ti, p]], K).astype(np.float64)          # [rows][K]
            rows = w.shape[0]
            wx = (w * x[ti][None, :]).reshape(rows, K // 32, 32).sum(axis=2)
            if off:
                blk = W[ids[ti, p]].reshape(rows, K // 32, -1)
                dw = blk[:, :, :2].copy().view(np.float16)[..., 0].astype(np.float64)   # [rows][K/32]
                u = w + off * np.repeat(dw, 32, axis=1)
                ux = (u * x[ti][None, :]).reshape(rows, K // 32, 32).sum(axis=2)
                xs = x[ti].reshape(K // 32, 32).sum(axis=1)
                v = (u ** 2) @ (step["q8_1"][0][ti] ** 2 / 12.0) + (w ** 2) @ (step["cpu"][0][ti] ** 2 / 12.0)
                v += ((ux ** 2).sum(axis=1) + (wx ** 2).sum(axis=1)) * f16
                v += ((off * dw) ** 2 * xs[None, :] ** 2).sum(axis=1) * f16
            else:
                v = (w ** 2) @ var_el[ti]
                v += (wx ** 2).sum(axis=1) * f16 * (2 if f16_cpu else 1)
            out[ti, p] = np.sqrt(v)
    return out
