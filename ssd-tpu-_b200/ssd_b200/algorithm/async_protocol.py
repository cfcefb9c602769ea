"""Async SSD request/response message types (jax_ssd/algorithm/async_protocol.py:11-40)."""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum

import torch


class DraftCommand(IntEnum):
    PREFILL = 0
    SERVE = 1
    SHUTDOWN = 2


@dataclass
class DraftRequest:
    command: DraftCommand
    cache_keys: torch.Tensor      # [B, 3] int32
    seq_lens: torch.Tensor        # [B] int32
    page_tables: torch.Tensor     # [B, max_pages] int32
    temperatures: torch.Tensor    # [B] float32
    prefix_tokens: list | None = None   # committed tokens per request (host)


@dataclass
class DraftResponse:
    cache_hit: torch.Tensor       # [B] bool
    spec_tokens: torch.Tensor     # [B, K] int32
    draft_logits: torch.Tensor    # [B, K, V] float32


@dataclass
class VerifyOutcome:
    seq_id: int
    accepted_length: int
    recovery_token: int

    def as_key(self) -> tuple[int, int, int]:
        return (self.seq_id, self.accepted_length, self.recovery_token)
