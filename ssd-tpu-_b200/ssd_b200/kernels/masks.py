"""Dense attention masks of the reference (jax_ssd/kernels/masks.py), for callers that build them.

The verify path does not use dense masks: the paged attention kernel applies
the verify visibility (full prefix + causal within the query tokens) from the
positions, and branch decoding gets the branch visibility from forked page
tables (``ssd_page_fork``).  These builders return the same additive fp32
masks (0 visible, -inf hidden) as device tensors.
"""

from __future__ import annotations

import torch


def _dev(device):
    return torch.device("cuda" if device is None else device)


def build_verify_mask(seq_len: int, query_len: int, device=None) -> torch.Tensor:
    """[query_len, seq_len + query_len]: query i sees the prefix and query tokens 0..i (masks.py:33-40)."""
    dev = _dev(device)
    q = torch.arange(query_len, device=dev)[:, None]
    k = torch.arange(seq_len + query_len, device=dev)[None, :]
    zero = torch.zeros((), dtype=torch.float32, device=dev)
    return torch.where(k < seq_len + q + 1, zero, torch.full((), float("-inf"), device=dev))


def build_branch_mask(batch: int, num_branches: int, trunk_len: int, branch_len: int, device=None) -> torch.Tensor:
    """[batch * num_branches, T, T], T = trunk_len + branch_len (masks.py:8-30): every query sees the
    trunk; a branch query also sees its own branch tokens up to itself."""
    dev = _dev(device)
    total = trunk_len + branch_len
    q = torch.arange(total, device=dev)[:, None]
    k = torch.arange(total, device=dev)[None, :]
    visible = (k < trunk_len) | ((q >= trunk_len) & (k >= trunk_len) & (k <= q))
    zero = torch.zeros((), dtype=torch.float32, device=dev)
    m = torch.where(visible, zero, torch.full((), float("-inf"), device=dev))
    return m.expand(batch * num_branches, total, total).contiguous()
