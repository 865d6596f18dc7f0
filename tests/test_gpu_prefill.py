"""Prefill MUL_MAT_ID (moe_b200_prefill_mul_mat_id) against the oracle's
llama.cpp CPU MUL_MAT_ID (Q8_K activations).

Q2_K on the tensor-core path computes each super-block's integer dot exactly
and finishes it with llama.cpp's own float steps in the same order, so the
result is compared bit for bit, as are Q4_0, Q5_0 and Q8_0 (per-block float
steps against Q8_0 activations). Q3_K, Q4_K, Q5_K and Q6_K also have exact integer
super-block dots but sum them in float once per super-block where llama.cpp
keeps 8 lane sums; those and the types without a tensor-core path (decode
GEMV, in-kernel Q8_K) are held to max |gpu - ref| / max |ref| <= 1e-4 per
output vector."""
import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, experts, rel_err, zipf_logits

pytestmark = pytest.mark.gpu

TIGHT = 1e-4


def _zipf_ids(n_tok, E, k, seed):
    """top-k of Zipf-skewed logits: distinct experts per token, a few hot experts"""
    lg = zipf_logits(n_tok, E, seed)
    return np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)


def _run(pkg, cuda, t, W, K, rows, x, ids):
    mc = pkg.moe_cache
    Wd = torch.from_numpy(W).to(cuda)
    src0 = mc.expert_tensor(Wd, t, K, rows, name="w")
    dst, tc = mc.prefill_mul_mat_id(src0, torch.from_numpy(x).to(cuda), torch.from_numpy(ids).to(cuda))
    torch.cuda.synchronize()
    assert mc.device_error() == 0
    return dst.cpu().numpy(), tc


@pytest.mark.parametrize("K,rows,E,k,n_tok,seed", [
    (256, 128, 4, 1, 1, 1),          # one super-block, one token: 1 of a chunk's 64 token slots
    (768, 256, 8, 2, 100, 2),        # odd super-block count, ragged token chunks
    (1024, 384, 16, 4, 130, 3),      # 130 tokens: chunks of 64 + 64 + 2 on the hot experts
    (3072, 768, 32, 8, 64, 4),       # config-2 gate/up shape (1008-byte rows: the widest packed tile)
    (768, 3072, 32, 8, 48, 5),       # config-2 down shape (24 row blocks)
])
def test_prefill_q2k_tensor_cores_bit_exact(pkg, cuda, K, rows, E, k, n_tok, seed):
    W = experts(O.Q2_K, E, rows, K, seed)
    x = activations((n_tok, K), seed + 10)
    ids = _zipf_ids(n_tok, E, k, seed + 20)
    got, tc = _run(pkg, cuda, O.Q2_K, W, K, rows, x, ids)
    assert tc
    ref = O.mul_mat_id(O.Q2_K, W, K, x[:, None, :], ids)
    np.testing.assert_array_equal(got, ref)


def test_prefill_q2k_all_tokens_one_expert(pkg, cuda):
    """every pick on one expert (many chunks of one expert), others idle"""
    K, rows, E, k, n_tok = 512, 256, 8, 1, 200
    W = experts(O.Q2_K, E, rows, K, 7)
    x = activations((n_tok, K), 8)
    ids = np.full((n_tok, k), 5, dtype=np.int32)
    got, tc = _run(pkg, cuda, O.Q2_K, W, K, rows, x, ids)
    assert tc
    np.testing.assert_array_equal(got, O.mul_mat_id(O.Q2_K, W, K, x[:, None, :], ids))


def test_prefill_q2k_repeat_same_result(pkg, cuda):
    """entry order inside an expert comes from atomics; results must not depend on it"""
    K, rows, E, k, n_tok = 512, 128, 4, 4, 96
    W = experts(O.Q2_K, E, rows, K, 9)
    x = activations((n_tok, K), 10)
    ids = _zipf_ids(n_tok, E, k, 11)
    a, _ = _run(pkg, cuda, O.Q2_K, W, K, rows, x, ids)
    b, _ = _run(pkg, cuda, O.Q2_K, W, K, rows, x, ids)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("t,K,rows,E,k,n_tok,seed", [
    (O.Q3_K, 256, 128, 4, 1, 1, 21),
    (O.Q3_K, 768, 256, 8, 2, 100, 22),     # 330-byte rows: 8-row tensor-map groups, 2-byte aligned blocks
    (O.Q3_K, 3072, 768, 32, 8, 64, 23),
    (O.Q4_K, 512, 128, 8, 2, 70, 24),      # 70 tokens on the hot expert: chunks of 64 + 6
    (O.Q4_K, 3072, 768, 32, 8, 64, 25),
    (O.Q4_K, 768, 3072, 32, 8, 48, 26),
    (O.Q6_K, 256, 128, 4, 1, 33, 27),
    (O.Q6_K, 768, 256, 8, 2, 100, 28),     # 630-byte rows
    (O.Q6_K, 3072, 768, 32, 8, 64, 29),
    (O.Q5_K, 256, 128, 4, 1, 1, 30),
    (O.Q5_K, 512, 128, 8, 2, 70, 31),      # chunks of 64 + 6 on the hot expert
    (O.Q5_K, 3072, 768, 32, 8, 64, 32),
    (O.Q5_K, 768, 3072, 32, 8, 48, 33),
])
def test_prefill_kquants_tensor_cores(pkg, cuda, t, K, rows, E, k, n_tok, seed):
    """Q3_K / Q4_K / Q5_K / Q6_K on the tensor cores: exact integer dots,
    llama.cpp's float steps up to the order of the sub-block sums"""
    W = experts(t, E, rows, K, seed)
    x = activations((n_tok, K), seed + 10)
    ids = _zipf_ids(n_tok, E, k, seed + 20)
    got, tc = _run(pkg, cuda, t, W, K, rows, x, ids)
    assert tc
    assert rel_err(got, O.mul_mat_id(t, W, K, x[:, None, :], ids)) <= TIGHT


@pytest.mark.parametrize("t,K,rows,E,k,n_tok,seed", [
    (O.Q4_0, 32 * 8, 128, 4, 1, 1, 41),      # one step, one token
    (O.Q4_0, 2048, 512, 16, 4, 70, 42),      # config-1 gate/up shape, chunks of 16 + ragged
    (O.Q4_0, 512, 2048, 16, 4, 40, 43),      # config-1 down shape
    (O.Q5_0, 768, 256, 8, 2, 100, 44),
    (O.Q5_0, 3072, 768, 32, 8, 64, 45),
    (O.Q8_0, 128, 128, 4, 1, 5, 46),         # one 128-value step
    (O.Q8_0, 1024, 384, 8, 2, 33, 47),
    (O.Q8_0, 3072, 768, 32, 8, 64, 48),
])
def test_prefill_block32_tensor_cores_bit_exact(pkg, cuda, t, K, rows, E, k, n_tok, seed):
    """Q4_0 / Q5_0 / Q8_0 on the tensor cores against Q8_0 activations: exact
    integer block dots, llama.cpp's per-block float steps in block order --
    equal to the CPU path bit for bit"""
    W = experts(t, E, rows, K, seed)
    x = activations((n_tok, K), seed + 10)
    ids = _zipf_ids(n_tok, E, k, seed + 20)
    got, tc = _run(pkg, cuda, t, W, K, rows, x, ids)
    assert tc
    np.testing.assert_array_equal(got, O.mul_mat_id(t, W, K, x[:, None, :], ids))


@pytest.mark.parametrize("t,K,rows", [(O.Q4_0, 256, 96), (O.Q8_0, 256, 100),
                                      (O.Q2_K, 256, 192), (O.Q5_K, 512, 200)])   # rows not a multiple of 128
def test_prefill_fallback_gemv(pkg, cuda, t, K, rows):
    E, k, n_tok = 8, 2, 19
    W = experts(t, E, rows, K, 12)
    x = activations((n_tok, K), 13)
    ids = _zipf_ids(n_tok, E, k, 14)
    got, tc = _run(pkg, cuda, t, W, K, rows, x, ids)
    assert not tc
    assert rel_err(got, O.mul_mat_id(t, W, K, x[:, None, :], ids)) <= TIGHT


def test_prefill_bad_id_reported(pkg, cuda):
    """an out-of-range expert id is skipped and reported as a device error"""
    K, rows, E, k, n_tok = 256, 128, 4, 2, 8
    W = experts(O.Q2_K, E, rows, K, 15)
    x = activations((n_tok, K), 16)
    ids = _zipf_ids(n_tok, E, k, 17)
    ids[3, 1] = E + 7
    mc = pkg.moe_cache
    src0 = mc.expert_tensor(torch.from_numpy(W).to(cuda), O.Q2_K, K, rows)
    mc.prefill_mul_mat_id(src0, torch.from_numpy(x).to(cuda), torch.from_numpy(ids).to(cuda))
    torch.cuda.synchronize()
    assert mc.device_error() != 0


@pytest.mark.parametrize("t", [O.Q2_K, O.Q4_0, O.Q6_K])
def test_prefill_tiered_pool_on_tensor_cores(pkg, cuda, tmp_path, t):
    """A host-tiered tensor (pinned host memory, a pool of 4 slots seeded with
    4 experts): picks of pool-resident experts run on the tensor cores with
    the pool as the expert array, the other picks through the GEMV reading
    host memory in place; together equal to the oracle."""
    mc = pkg.moe_cache
    K, rows, E, k, n_tok = 512, 256, 16, 2, 64
    W = experts(t, E, rows, K, 51)
    name = "blk.0.ffn_up_exps.weight"
    seed = tmp_path / "seed.txt"
    seed.write_text(f"{name} 3,1,4,5,9,2\n")
    mc.reset()
    mc.configure(enabled=True, slots=4, budget_gb=1.0, seed_path=str(seed))
    try:
        buf = torch.from_numpy(W).pin_memory()
        src0 = mc.expert_tensor(buf, t, K, rows, name=name)
        assert mc.wants(src0)
        x = activations((n_tok, K), 52)
        ids = _zipf_ids(n_tok, E, k, 53)
        dst, tc = mc.prefill_mul_mat_id(src0, torch.from_numpy(x).to(cuda), torch.from_numpy(ids).to(cuda))
        torch.cuda.synchronize()
        assert mc.device_error() == 0
        assert tc
        tbl, n_slots, _ = mc.table(src0)
        assert n_slots == 4 and sum(1 for v in tbl if v >= 0) == 4
        picks = ids.reshape(-1)
        assert any(tbl[e] >= 0 for e in picks) and any(tbl[e] == -1 for e in picks)
        ref = O.mul_mat_id(t, W, K, x[:, None, :], ids)
        assert rel_err(dst.cpu().numpy(), ref) <= TIGHT
    finally:
        mc.reset()
        mc.configure(enabled=True)
