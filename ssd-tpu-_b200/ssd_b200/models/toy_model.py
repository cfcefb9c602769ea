"""Context-free toy model with the reference's numbers (replaces jax_ssd/models/toy_model.py).

The reference's ``ToyModelAdapter`` (toy_model.py:13-41) gives token ``t`` the
logits ``h(t) @ W``, where ``h(t)`` is zero except ``h[t % H] = 1.0`` and then
``h[(7 t) % H] = 0.5`` (the second write wins when both indices coincide) and
``W`` is ``default_rng(seed).standard_normal((H, V)) * 0.1`` in fp32.  The
logits of a token therefore depend only on ``t mod H``: they are one of H rows.
This adapter builds those H rows once, with the reference's own fp32
expression (two non-zero terms per dot product, so every row is the single
rounding of ``W[a] + 0.5 W[b]`` whatever the summation order), and keeps them
on the device.  Every forward is then a row gather on the device
(``ssd_embed``), and draft tokens come from ``ssd_argmax_rows``.  It has no
layers, attention or KV writes, like the reference; ``allocate_kv`` still
returns a cache of the reference's shape for callers that pass one around.

``ssd_embed`` scales each gathered row by sqrt(row width).  The table is stored
pre-divided by that factor with a row width padded to a power of 4, so the
factor is a power of 2 and both the division and the kernel's multiplication
are exact: the device logits equal the reference's bit for bit.

The Gemma-style toy pair that the engine selects with ``SSD_USE_TOY_MODEL`` is
a different model (``models.gemma.PRESETS["toy-target"]``); this class is for
callers that construct the reference's lookup toy directly.
"""

from __future__ import annotations

import numpy as np
import torch

from ..algorithm.verify import argmax_rows
from ..kernels.kv_cache import KVCacheState
from ..kernels.ops import embed
from .base import DecodeResult, PrefillResult, VerifyResultModel


def toy_logit_rows(vocab_size: int, hidden_dim: int, seed: int) -> np.ndarray:
    """The H distinct logit rows [H, V] fp32 of the reference toy (row r serves every t with t % H == r)."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((hidden_dim, vocab_size)).astype(np.float32) * 0.1
    h = np.zeros((hidden_dim, hidden_dim), dtype=np.float32)
    for r in range(hidden_dim):
        h[r, r % hidden_dim] = 1.0
        h[r, (r * 7) % hidden_dim] = 0.5
    return (h @ w).astype(np.float32)


class ToyModelAdapter:
    """Deterministic lookup LM on the device: logits depend on the token id alone."""

    def __init__(self, vocab_size: int = 64, hidden_dim: int = 32, num_layers: int = 2, num_blocks: int = 32,
                 block_size: int = 16, seed: int = 0, device=None) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("ToyModelAdapter runs on the CUDA library and needs a CUDA device")
        self.vocab_size = vocab_size
        self.hidden_dim = hidden_dim
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        rows = toy_logit_rows(vocab_size, hidden_dim, seed)
        width = 1
        while width < vocab_size:
            width *= 4
        self._width = width
        scale = np.float32(np.sqrt(np.float32(width)))  # a power of 2, as ssd_embed computes it
        table = np.zeros((hidden_dim, width), dtype=np.float32)
        table[:, :vocab_size] = rows / scale
        self._table = torch.from_numpy(table).to(self.dev)

    # ------------------------------------------------------------ device forward
    def _logits(self, token_ids) -> torch.Tensor:
        """Logits [n, V] fp32 of the tokens, gathered on the device."""
        ids = torch.as_tensor(token_ids, dtype=torch.int64).reshape(-1).to(self.dev)
        if ids.numel() == 0:
            return torch.empty((0, self.vocab_size), dtype=torch.float32, device=self.dev)
        res = torch.remainder(ids, self.hidden_dim).to(torch.int32)
        out = embed(res, self._table)  # [n, width], exact rows
        return out if self._width == self.vocab_size else out[:, :self.vocab_size].contiguous()

    def _argmax(self, logits: torch.Tensor) -> int:
        nxt = torch.empty(1, dtype=torch.int32, device=self.dev)
        argmax_rows(logits[-1:], nxt)
        return int(nxt.item())

    # ------------------------------------------------------------ protocol
    def allocate_kv(self) -> KVCacheState:
        return KVCacheState.allocate(self.num_layers, self.num_blocks, self.block_size, 1, self.hidden_dim,
                                     device=self.dev)

    def prefill(self, token_ids, kv_cache=None, page_table=None) -> PrefillResult:
        """Logits of every prompt position, [len, V] (toy_model.py:52-59)."""
        return PrefillResult(logits=self._logits(token_ids), kv_cache=kv_cache)

    def decode(self, token_id: int, position: int | None = None, kv_cache=None, page_table=None) -> DecodeResult:
        lg = self._logits([int(token_id)])
        return DecodeResult(logits=lg, kv_cache=kv_cache, next_token=self._argmax(lg))

    def verify(self, token_ids_kp1, positions=None, kv_cache=None, page_table=None) -> VerifyResultModel:
        """Logits [1, K+1, V] fp32 of the k+1 tokens (toy_model.py:72-80)."""
        return VerifyResultModel(logits=self._logits(token_ids_kp1)[None], kv_cache=kv_cache)

    def draft_speculate(self, prefix_tokens: list[int], k: int) -> tuple[list[int], torch.Tensor]:
        """k greedy tokens after the prefix and the logits that chose them, [k, V] (toy_model.py:82-96)."""
        tokens = [int(t) for t in prefix_tokens]
        logits = torch.empty((k, self.vocab_size), dtype=torch.float32, device=self.dev)
        for i in range(k):
            lg = self._logits(tokens[-1:])
            logits[i].copy_(lg[0])
            tokens.append(self._argmax(lg))
        return tokens[len(prefix_tokens):], logits

    def commit_tokens(self, token_ids: list[int]) -> None:
        return

    def tokenize(self, text: str) -> list[int]:
        return [ord(c) % self.vocab_size for c in text]

    def decode_tokens_to_str(self, token_ids: list[int]) -> str:
        return " ".join(f"t{int(t)}" for t in token_ids)
