"""Oracle: paged KV layout, slot writes and multi-query verify attention (test infrastructure only).

Restates, from the reference:

* page layout ``[2, num_layers, num_blocks, block_size, num_kv_heads, head_dim]``
  — ``jax_ssd/kernels/kv_cache.py:13,28-31`` (plane 0 = K, plane 1 = V);
* ``write_kv_slots`` — kv_cache.py:39-58 (``block = slot // bs``,
  ``offset = slot % bs``), with the slot of position ``p`` of a sequence being
  ``block_table[p // bs] * bs + p % bs`` (the indexing of kv_cache.py:68);
* ``build_verify_mask`` — ``jax_ssd/kernels/masks.py:33-40``: query ``i`` of a
  block of ``T`` new tokens sees the whole prefix plus new tokens ``0..i``;
* ``masked_dot_product_attention`` — ``jax_ssd/kernels/attention_ref.py:9-21``:
  ``softmax(q k^T / sqrt(d) + mask) v``.

Parity unpinned (the reference never runs these on the model path and its JAX
code cannot be imported here).
"""

from __future__ import annotations

import numpy as np


def slot_of(block_table: np.ndarray, pos: np.ndarray, block_size: int) -> np.ndarray:
    return block_table[pos // block_size] * block_size + pos % block_size


def write_kv(pages, layer, block_tables, positions, k, v):
    """pages[2,L,NB,BS,H,D]; block_tables[B,M]; positions[B,T] (-1 = skip); k,v[B,T,H,D]."""
    bs = pages.shape[3]
    for b in range(positions.shape[0]):
        for t in range(positions.shape[1]):
            p = int(positions[b, t])
            if p < 0:
                continue
            blk = int(block_tables[b, p // bs])
            pages[0, layer, blk, p % bs] = k[b, t]
            pages[1, layer, blk, p % bs] = v[b, t]
    return pages


def verify_mask(seq_len: int, query_len: int) -> np.ndarray:
    """masks.py:33-40."""
    m = np.full((query_len, seq_len + query_len), -np.inf, np.float32)
    m[:, :seq_len] = 0.0
    for i in range(query_len):
        m[i, seq_len : seq_len + i + 1] = 0.0
    return m


def branch_mask(batch: int, num_branches: int, trunk_len: int, branch_len: int) -> np.ndarray:
    """masks.py:8-30: every query sees the trunk; branch query i sees branch tokens 0..i."""
    total = trunk_len + branch_len
    m = np.full((batch * num_branches, total, total), -np.inf, np.float32)
    for b in range(batch * num_branches):
        m[b, :, :trunk_len] = 0.0
        for i in range(branch_len):
            m[b, trunk_len + i, trunk_len : trunk_len + i + 1] = 0.0
    return m


def attention_ref(q, k, v, mask):
    """attention_ref.py:9-21 in float64 (q[...,Tq,D], k/v[...,Tk,D])."""
    d = q.shape[-1]
    s = np.einsum("...qd,...kd->...qk", q.astype(np.float64), k.astype(np.float64)) / np.sqrt(d)
    s = s + mask
    s = s - s.max(-1, keepdims=True)
    w = np.exp(s)
    w /= w.sum(-1, keepdims=True)
    return np.einsum("...qk,...kd->...qd", w, v.astype(np.float64))


def paged_verify_attention(q, pages, layer, block_tables, seq_lens, q_lens=None):
    """Multi-query attention of the new tokens against their sequence's pages.

    q[B,T,Hq,D]; seq_lens[B] = cached tokens INCLUDING the new ones; q_lens[B]
    (default T) = valid new tokens (rows t >= q_lens[b] are left zero).
    Query t sits at position seq_lens[b] - q_lens[b] + t.  GQA: head h reads KV
    head h // (Hq // Hkv).  Returns float64 [B,T,Hq,D].
    """
    bsz, tq, hq, d = q.shape
    bs = pages.shape[3]
    hkv = pages.shape[4]
    g = hq // hkv
    out = np.zeros((bsz, tq, hq, d), np.float64)
    for b in range(bsz):
        n = int(seq_lens[b])
        ql = tq if q_lens is None else int(q_lens[b])
        if n == 0 or ql == 0:
            continue
        pos = np.arange(n)
        blk = block_tables[b, pos // bs]
        kk = pages[0, layer, blk, pos % bs].astype(np.float64)  # [n,Hkv,D]
        vv = pages[1, layer, blk, pos % bs].astype(np.float64)
        mask = verify_mask(n - ql, ql)
        for h in range(hq):
            out[b, :ql, h] = attention_ref(q[b, :ql, h], kk[:, h // g], vv[:, h // g], mask)
    return out
