"""Model adapter interface (jax_ssd/models/base.py:14-60), on torch device tensors."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch

from ..kernels.kv_cache import KVCacheState


@dataclass
class PrefillResult:
    logits: torch.Tensor            # [1, V]: the last prompt position
    kv_cache: KVCacheState
    hidden_states: torch.Tensor | None = None


@dataclass
class DecodeResult:
    logits: torch.Tensor            # [1, V]
    kv_cache: KVCacheState
    next_token: int


@dataclass
class VerifyResultModel:
    logits: torch.Tensor            # [B, K+1, V] fp32
    kv_cache: KVCacheState


class DecodeModelAdapter(Protocol):
    vocab_size: int

    def prefill(self, token_ids, kv_cache: KVCacheState, page_table) -> PrefillResult: ...

    def decode(self, token_id: int, position: int, kv_cache: KVCacheState, page_table) -> DecodeResult: ...

    def verify(self, token_ids_kp1, positions, kv_cache: KVCacheState, page_table) -> VerifyResultModel: ...

    def decode_tokens_to_str(self, token_ids: list[int]) -> str: ...
