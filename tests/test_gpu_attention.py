"""GPU parity: paged multi-query verify attention (K1) and KV writes (K2) vs the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.gemma import bf16_round
from oracle.paged_kv import paged_verify_attention as o_attn
from oracle.paged_kv import write_kv as o_write

pytestmark = pytest.mark.gpu


def _setup(b, t, hq, hkv, d, bs, ctx, dtype_name, seed, table_cols=None):
    import torch

    from ssd_b200.kernels.kv_cache import KVCacheState

    rng = np.random.default_rng(seed)
    max_blocks = max((c + bs - 1) // bs for c in ctx)
    nb = b * max_blocks + 3
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.full((b, max_blocks), -1, np.int32)
    for i, c in enumerate(ctx):
        nbk = (c + bs - 1) // bs
        tables[i, :nbk] = perm[i * max_blocks: i * max_blocks + nbk]
    tdt = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    cache = KVCacheState.allocate(1, nb, bs, hkv, d, dtype=tdt)
    pages_np = np.zeros((2, 1, nb, bs, hkv, d), np.float32)
    L = max(ctx)
    k = rng.standard_normal((b, L, hkv, d)).astype(np.float32)
    v = rng.standard_normal((b, L, hkv, d)).astype(np.float32)
    q = rng.standard_normal((b, t, hq, d)).astype(np.float32)
    if dtype_name == "bf16":
        k, v, q = bf16_round(k), bf16_round(v), bf16_round(q)
    pos = np.where(np.arange(L)[None, :] < np.array(ctx)[:, None], np.arange(L)[None, :], -1).astype(np.int32)
    o_write(pages_np, 0, tables, pos, k, v)
    cache.pages.copy_(torch.tensor(pages_np).to(tdt))
    if table_cols is not None and table_cols > tables.shape[1]:  # unused trailing entries stay -1
        tables = np.concatenate([tables, np.full((b, table_cols - tables.shape[1]), -1, np.int32)], 1)
    return cache, pages_np, tables, q, tdt


@pytest.mark.parametrize("dtype_name,hq,hkv,d,t,bs,b,lo,hi,tol", [
    ("bf16", 16, 16, 256, 5, 16, 8, 512, 4096, 2e-2),   # op config 2a (Gemma-7B verify attention)
    ("bf16", 8, 1, 256, 1, 16, 3, 1, 700, 2e-2),       # Gemma-2B draft decode (MQA)
    ("bf16", 8, 1, 256, 3, 16, 2, 40, 300, 2e-2),      # G*T = 24 rows -> two row groups
    ("bf16", 2, 2, 256, 5, 16, 4, 300, 2000, 2e-2),    # Gemma-7B shard at 8 ranks (6-consumer variant)
    ("f32", 4, 1, 64, 5, 16, 4, 5, 200, 1e-5),         # toy pair, fp32
    ("f32", 4, 2, 128, 7, 4, 3, 7, 90, 1e-5),          # small pages, k = 6
])
def test_paged_attention_matches_oracle(cuda, dtype_name, hq, hkv, d, t, bs, b, lo, hi, tol):
    import torch

    from ssd_b200.kernels.kv_cache import paged_verify_attention

    rng = np.random.default_rng(hq * d + t)
    ctx = [int(c) for c in rng.integers(max(lo, t), hi + 1, b)]
    cache, pages_np, tables, q, tdt = _setup(b, t, hq, hkv, d, bs, ctx, dtype_name, seed=b + t)
    tb = torch.tensor(tables, device="cuda")
    sl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    out = paged_verify_attention(torch.tensor(q).to(device="cuda", dtype=tdt), cache, 0, tb, sl,
                                 max_seq_len=tables.shape[1] * bs)
    ref = o_attn(q, pages_np, 0, tables, np.array(ctx))
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, atol=tol, rtol=tol)


def test_ragged_q_lens_and_padding_rows(cuda):
    import torch

    from ssd_b200.kernels.kv_cache import paged_verify_attention

    b, t, hq, hkv, d, bs = 4, 5, 4, 2, 64, 16
    ctx = [5, 40, 200, 17]
    ql = np.array([5, 2, 0, 1], np.int32)
    cache, pages_np, tables, q, tdt = _setup(b, t, hq, hkv, d, bs, ctx, "f32", seed=3)
    out = paged_verify_attention(torch.tensor(q, device="cuda"), cache, 0, torch.tensor(tables, device="cuda"),
                                 torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                                 q_lens=torch.tensor(ql, device="cuda"), max_seq_len=tables.shape[1] * bs)
    ref = o_attn(q, pages_np, 0, tables, np.array(ctx), q_lens=ql)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-5, rtol=1e-5)
    assert (out[2] == 0).all() and (out[1, 2:] == 0).all()


@pytest.mark.parametrize("hq,hkv", [(16, 16), (8, 1), (8, 2)])
def test_attention_is_batch_invariant(cuda, hq, hkv):
    """A query's output is bit-identical whether it is verified with k others or decoded alone."""
    import torch

    from ssd_b200.kernels.kv_cache import paged_verify_attention

    b, t, d, bs = 1, 5, 256, 16
    ctx = [777]
    cache, pages_np, tables, q, tdt = _setup(b, t, hq, hkv, d, bs, ctx, "bf16", seed=9, table_cols=128)
    tb = torch.tensor(tables, device="cuda")
    qd = torch.tensor(q).to(device="cuda", dtype=tdt)
    full = paged_verify_attention(qd, cache, 0, tb, torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                                  max_seq_len=2048)
    for i in range(t):
        n = ctx[0] - t + i + 1
        one = paged_verify_attention(qd[:, i:i + 1].contiguous(), cache, 0, tb,
                                     torch.tensor([n], dtype=torch.int32, device="cuda"), max_seq_len=1024)
        assert torch.equal(one[0, 0], full[0, i])


def test_kv_write_and_slots(cuda):
    import torch

    from ssd_b200.kernels.kv_cache import KVCacheState, write_kv, write_kv_slots

    rng = np.random.default_rng(4)
    nl, nb, bs, h, d = 3, 10, 4, 2, 64
    cache = KVCacheState.allocate(nl, nb, bs, h, d, dtype=torch.bfloat16)
    tables = rng.permutation(nb).astype(np.int32).reshape(2, 5)
    pos = np.array([[0, 5, 19, -1], [3, 4, 7, 12]], np.int32)
    k = bf16_round(rng.standard_normal((2, 4, h, d)).astype(np.float32))
    v = bf16_round(rng.standard_normal((2, 4, h, d)).astype(np.float32))
    write_kv(cache, 1, torch.tensor(tables, device="cuda"), torch.tensor(pos, device="cuda"),
             torch.tensor(k).cuda().bfloat16(), torch.tensor(v).cuda().bfloat16())
    exp = np.zeros((2, nl, nb, bs, h, d), np.float32)
    o_write(exp, 1, tables, pos, k, v)
    np.testing.assert_array_equal(cache.pages.float().cpu().numpy(), exp)
    # write_kv_slots: slot s -> block s // bs, offset s % bs (kv_cache.py:39-58)
    slots = np.array([0, 7, 39], np.int32)
    kk = torch.ones((3, h, d), dtype=torch.bfloat16, device="cuda")
    write_kv_slots(cache, 2, torch.tensor(slots, device="cuda"), kk, 2 * kk)
    p = cache.pages.float().cpu().numpy()
    for s in slots:
        assert (p[0, 2, s // bs, s % bs] == 1).all() and (p[1, 2, s // bs, s % bs] == 2).all()
