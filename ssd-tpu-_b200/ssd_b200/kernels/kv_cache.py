"""Paged KV cache on the GPU (drop-in for jax_ssd/kernels/kv_cache.py).

Layout kept from the reference (kv_cache.py:13,28-31):
``pages[2, num_layers, num_blocks, block_size, num_kv_heads, head_dim]``
(plane 0 = K, plane 1 = V).  Writes and attention run in the K1/K2 kernels.
Unlike the functional JAX original (which returns a new array), writes update
``pages`` in place; the returned ``KVCacheState`` aliases the same storage.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .._lib import check, dtype_code, lib, ptr, stream_ptr
from ..workspace import workspace


@dataclass
class KVCacheState:
    """Paged KV cache: [2, num_layers, num_blocks, block_size, num_kv_heads, head_dim]."""

    pages: torch.Tensor
    block_size: int

    @classmethod
    def allocate(cls, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype=torch.bfloat16, device="cuda") -> "KVCacheState":
        pages = torch.zeros((2, num_layers, num_blocks, block_size, num_kv_heads, head_dim), dtype=dtype,
                            device=device)
        return cls(pages=pages, block_size=block_size)

    @property
    def num_blocks(self) -> int:
        return self.pages.shape[2]

    @property
    def num_layers(self) -> int:
        return self.pages.shape[1]


def _dims(cache: KVCacheState):
    _, nl, nb, bs, hkv, hd = cache.pages.shape
    return nl, nb, bs, hkv, hd


def gather_kv_for_positions(cache: KVCacheState, layer: int, page_table, positions) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V rows [n, num_kv_heads, head_dim] of one sequence's positions (kv_cache.py:61-72).

    Slot of position p: page_table[p // block_size] * block_size + p % block_size, as in the
    reference.  The reference computes the slots and returns zeros (its gather is a stub);
    this returns the stored rows, in the cache's dtype.
    """
    dev = cache.pages.device
    pt = torch.as_tensor(page_table).to(dev).long().reshape(-1)
    pos = torch.as_tensor(positions).to(dev).long().reshape(-1)
    blk = pt[pos // cache.block_size]
    off = pos % cache.block_size
    return cache.pages[0, layer, blk, off], cache.pages[1, layer, blk, off]


def write_kv(cache: KVCacheState, layer: int, block_tables: torch.Tensor, positions: torch.Tensor,
             k: torch.Tensor, v: torch.Tensor) -> KVCacheState:
    """K2: write k/v [B,T,Hkv,D] at positions [B,T] (-1 = skip) through block_tables [B,M]."""
    nl, nb, bs, hkv, hd = _dims(cache)
    b, t = positions.shape
    check(lib().ssd_kv_write(stream_ptr(), ptr(cache.pages), dtype_code(cache.pages.dtype), nl, nb, bs, hkv, hd,
                             layer, ptr(block_tables), block_tables.shape[1], ptr(positions), ptr(k.contiguous()),
                             ptr(v.contiguous()), b, t), "ssd_kv_write")
    return cache


def write_kv_slots(cache: KVCacheState, layer: int, slot_mapping: torch.Tensor, k: torch.Tensor,
                   v: torch.Tensor) -> KVCacheState:
    """kv_cache.py:39-58: slot s goes to block s // bs, offset s % bs."""
    nl, nb, bs, hkv, hd = _dims(cache)
    dev = cache.pages.device
    ident = torch.arange(nb, dtype=torch.int32, device=dev)[None, :]
    slots = torch.as_tensor(slot_mapping).to(device=dev, dtype=torch.int32).reshape(1, -1)
    n = slots.shape[1]
    return write_kv(cache, layer, ident, slots, k.reshape(1, n, hkv, hd), v.reshape(1, n, hkv, hd))


def paged_verify_attention(q: torch.Tensor, cache: KVCacheState, layer: int, block_tables: torch.Tensor,
                           seq_lens: torch.Tensor, q_lens: torch.Tensor | None = None,
                           scale: float | None = None, max_seq_len: int | None = None,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """K1: attention of q [B,T,Hq,D] against each sequence's pages.

    seq_lens [B] counts cached tokens INCLUDING the new ones; new token t of
    sequence b sits at position seq_lens[b] - q_lens[b] + t (masks.py:33-40).
    """
    nl, nb, bs, hkv, hd = _dims(cache)
    b, t, hq, d = q.shape
    if d != hd:
        raise ValueError("head_dim mismatch")
    if max_seq_len is None:
        max_seq_len = block_tables.shape[1] * bs
    if scale is None:
        scale = 1.0 / float(hd) ** 0.5
    if out is None:
        out = torch.empty_like(q)
    nbytes = lib().ssd_paged_attention_workspace_size(b, t, hq, hkv, hd, max_seq_len)
    ws = workspace(q.device, "paged_attention", nbytes)
    check(lib().ssd_paged_verify_attention(stream_ptr(), ptr(q.contiguous()), ptr(cache.pages),
                                           dtype_code(cache.pages.dtype), nl, nb, bs, hkv, hd, layer,
                                           ptr(block_tables), block_tables.shape[1], ptr(seq_lens), ptr(q_lens),
                                           ptr(out), float(scale), b, t, hq, int(max_seq_len), ptr(ws), ws.numel()),
          "ssd_paged_verify_attention")
    return out
