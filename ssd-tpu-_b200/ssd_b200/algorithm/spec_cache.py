"""Tensor-backed draft speculation cache (drop-in for jax_ssd/algorithm/spec_cache.py).

Same fields and methods as the reference (``create/reset/lookup/insert/
insert_batch``); ``lookup`` runs the ``ssd_spec_cache_lookup`` kernel (first
valid slot whose [seq_id, accepted_index, recovery_token] key matches).  Unlike
the functional JAX original, inserts write the device tensors in place and
return ``self``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .._lib import check, lib, ptr, stream_ptr


@dataclass
class SpecCache:
    keys: torch.Tensor     # [N, 3] int32
    tokens: torch.Tensor   # [N, K] int32
    logits: torch.Tensor   # [N, K, V] float32
    valid: torch.Tensor    # [N] bool (uint8 storage)
    k: int
    vocab: int

    @classmethod
    def create(cls, num_branches: int, k: int, vocab: int, device="cuda", with_logits: bool = True) -> "SpecCache":
        dev = torch.device(device)
        return cls(keys=torch.zeros((num_branches, 3), dtype=torch.int32, device=dev),
                   tokens=torch.zeros((num_branches, k), dtype=torch.int32, device=dev),
                   logits=torch.zeros((num_branches if with_logits else 1, k, vocab), dtype=torch.float32, device=dev),
                   valid=torch.zeros((num_branches,), dtype=torch.uint8, device=dev), k=k, vocab=vocab)

    def reset(self) -> "SpecCache":
        self.valid.zero_()
        return self

    def lookup(self, request_keys) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """request_keys [B, 3] -> (hit [B] bool, idx [B] int32 (-1 on a miss), tokens [B, K], logits [B, K, V])."""
        req = torch.as_tensor(request_keys).to(device=self.keys.device, dtype=torch.int32).reshape(-1, 3).contiguous()
        b = req.shape[0]
        hit = torch.empty(b, dtype=torch.uint8, device=req.device)
        idx = torch.empty(b, dtype=torch.int32, device=req.device)
        tok = torch.empty((b, self.k), dtype=torch.int32, device=req.device)
        with_logits = self.logits.shape[0] == self.keys.shape[0]
        lg = torch.empty((b, self.k, self.vocab), dtype=torch.float32, device=req.device) if with_logits else None
        check(lib().ssd_spec_cache_lookup(stream_ptr(), ptr(self.keys), ptr(self.valid), ptr(self.tokens),
                                          ptr(self.logits) if with_logits else None, self.keys.shape[0], self.k,
                                          self.vocab, ptr(req), b, ptr(hit), ptr(idx), ptr(tok), ptr(lg)),
              "ssd_spec_cache_lookup")
        if lg is None:
            lg = torch.zeros((b, self.k, self.vocab), dtype=torch.float32, device=req.device)
        return hit.bool(), idx, tok, lg

    def insert(self, slot: int, key, tokens, logits=None) -> "SpecCache":
        self.keys[slot] = torch.as_tensor(key, dtype=torch.int32, device=self.keys.device)
        self.tokens[slot] = torch.as_tensor(tokens, dtype=torch.int32, device=self.keys.device)
        if logits is not None and self.logits.shape[0] == self.keys.shape[0]:
            self.logits[slot] = torch.as_tensor(logits, dtype=torch.float32, device=self.keys.device)
        self.valid[slot] = 1
        return self

    def insert_batch(self, start_slot: int, keys, tokens, logits=None) -> "SpecCache":
        n = len(keys)
        for i in range(n):
            self.insert(start_slot + i, keys[i], tokens[i], None if logits is None else logits[i])
        return self
