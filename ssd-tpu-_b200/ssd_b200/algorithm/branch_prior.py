"""Saguaro branch prior (jax_ssd/algorithm/branch_prior.py:9-66) on torch device tensors."""

from __future__ import annotations

import torch


def top_f_recovery_tokens(glue_logits: torch.Tensor, fan_out: int) -> torch.Tensor:
    """[B, V] or [B, K+1, V] (last position used) -> top-F token ids [B, F] int32."""
    if glue_logits.dim() == 3:
        glue_logits = glue_logits[:, -1, :]
    return torch.topk(glue_logits, fan_out, dim=-1).indices.to(torch.int32)


def build_branch_keys(seq_ids, accepted_indices, recovery_tokens) -> torch.Tensor:
    return torch.stack([torch.as_tensor(seq_ids), torch.as_tensor(accepted_indices),
                        torch.as_tensor(recovery_tokens)], dim=-1).to(torch.int32)


def expand_fanout_branches(base_keys: torch.Tensor, fan_out_list: tuple[int, ...], recovery_candidates: torch.Tensor):
    """base_keys [B,3], fan_out_list (K+1), recovery_candidates [B, max_F] -> ([B*mq_len, 3], mq_len)."""
    mq_len = sum(fan_out_list)
    branches = []
    for acc_idx, fan in enumerate(fan_out_list):
        for f in range(fan):
            key = base_keys.clone()
            key[:, 1] = acc_idx
            if recovery_candidates.shape[1] > f:
                key[:, 2] = recovery_candidates[:, f]
            branches.append(key)
    if not branches:
        return base_keys, base_keys.shape[0]
    return torch.cat(branches, 0), mq_len
