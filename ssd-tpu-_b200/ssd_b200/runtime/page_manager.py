"""Paged KV block allocation with device-resident state (drop-in for jax_ssd/runtime/page_manager.py).

The host API of the reference stays (``allocate`` / ``allocate_draft`` /
``rollback_speculative`` / ``free_sequence``, page_manager.py:21-64, with the
``free_blocks`` list and ``ref_counts`` dict readable as before), but the state
lives on the GPU and every operation is one K5 kernel launch
(``ssd_page_allocate`` / ``ssd_page_rollback`` / ``ssd_page_free``):

* ``free_list[num_blocks]`` + ``free_top``: the reference's ``free_blocks`` list
  (index ``free_top-1`` is its last element, where pops and pushes happen);
* ``ref_counts[num_blocks]``: the dict, 0 meaning "absent";
* ``tables[max_seqs, max_blocks]`` / ``lens`` (and the draft pair): one row per
  sequence slot.

The per-sequence host calls synchronise to return the reference's Python
values and to keep ``Sequence.block_table`` current.  The batched
``*_rows`` calls used by the engine take device tensors and never synchronise.
"""

from __future__ import annotations

import torch

from .._lib import check, lib, ptr, stream_ptr
from .sequence import Sequence


class PageManager:
    def __init__(self, block_size: int, num_blocks: int, free_blocks: list[int] | None = None,
                 ref_counts: dict[int, int] | None = None, *, max_seqs: int = 64,
                 max_blocks_per_seq: int | None = None, device="cuda") -> None:
        self.block_size = int(block_size)
        self.num_blocks = int(num_blocks)
        self.max_seqs = int(max_seqs)
        self.max_blocks = int(max_blocks_per_seq or num_blocks)
        self.device = torch.device(device)
        dev = self.device
        fb = list(range(self.num_blocks)) if not free_blocks else [int(b) for b in free_blocks]
        self.free_list = torch.full((self.num_blocks,), -1, dtype=torch.int32, device=dev)
        if fb:
            self.free_list[: len(fb)] = torch.tensor(fb, dtype=torch.int32, device=dev)
        self.free_top = torch.tensor([len(fb)], dtype=torch.int32, device=dev)
        self.ref_counts_dev = torch.zeros(self.num_blocks, dtype=torch.int32, device=dev)
        for k, v in (ref_counts or {}).items():
            self.ref_counts_dev[int(k)] = int(v)
        self.tables = torch.full((self.max_seqs, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(self.max_seqs, dtype=torch.int32, device=dev)
        self.draft_tables = torch.full((self.max_seqs, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self.draft_lens = torch.zeros(self.max_seqs, dtype=torch.int32, device=dev)
        self._rows: dict[int, int] = {}

    # ------------------------------------------------------------ host views
    @property
    def free_blocks(self) -> list[int]:
        top = int(self.free_top.item())
        return [int(x) for x in self.free_list[:top].tolist()]

    @property
    def ref_counts(self) -> dict[int, int]:
        rc = self.ref_counts_dev.tolist()
        return {i: int(c) for i, c in enumerate(rc) if c != 0}

    def row(self, seq: Sequence) -> int:
        r = self._rows.get(seq.seq_id)
        if r is None:
            used = set(self._rows.values())
            r = next((i for i in range(self.max_seqs) if i not in used), None)
            if r is None:
                raise RuntimeError(f"all {self.max_seqs} sequence slots of the page manager are in use; "
                                   "free_sequence() releases a finished sequence's slot")
            self._rows[seq.seq_id] = r
            # adopt any blocks the host object already lists
            if seq.block_table:
                self.tables[r, : len(seq.block_table)] = torch.tensor(seq.block_table, dtype=torch.int32,
                                                                      device=self.device)
                self.lens[r] = len(seq.block_table)
            if seq.draft_block_table:
                self.draft_tables[r, : len(seq.draft_block_table)] = torch.tensor(
                    seq.draft_block_table, dtype=torch.int32, device=self.device)
                self.draft_lens[r] = len(seq.draft_block_table)
        return r

    def _sync_seq(self, seq: Sequence, r: int) -> None:
        n, dn = int(self.lens[r].item()), int(self.draft_lens[r].item())
        seq.block_table[:] = [int(x) for x in self.tables[r, :n].tolist()]
        seq.draft_block_table[:] = [int(x) for x in self.draft_tables[r, :dn].tolist()]

    def _scalar(self, v: int) -> torch.Tensor:
        return torch.tensor([int(v)], dtype=torch.int32, device=self.device)

    # ------------------------------------------------------ reference host API
    def allocate(self, seq: Sequence, num_tokens: int) -> bool:
        """page_manager.py:21-33."""
        r = self.row(seq)
        ok = torch.zeros(1, dtype=torch.uint8, device=self.device)
        self.allocate_rows(r, 1, self._scalar(seq.num_tokens), self._scalar(num_tokens), ok, draft=False)
        self._sync_seq(seq, r)
        return bool(ok.item())

    def allocate_draft(self, seq: Sequence, num_tokens: int) -> bool:
        """page_manager.py:35-47."""
        r = self.row(seq)
        ok = torch.zeros(1, dtype=torch.uint8, device=self.device)
        self.allocate_rows(r, 1, self._scalar(seq.num_tokens), self._scalar(num_tokens), ok, draft=True)
        self._sync_seq(seq, r)
        return bool(ok.item())

    def rollback_speculative(self, seq: Sequence, accepted_tokens: int, reserved: int) -> None:
        """page_manager.py:49-56 (``reserved`` has no effect there either)."""
        r = self.row(seq)
        self.rollback_rows(r, 1, self._scalar(seq.num_tokens), self._scalar(accepted_tokens))
        self._sync_seq(seq, r)

    def free_sequence(self, seq: Sequence) -> None:
        """page_manager.py:58-64; the sequence's device slot is released too."""
        r = self.row(seq)
        rel = torch.ones(1, dtype=torch.uint8, device=self.device)
        check(lib().ssd_page_free(stream_ptr(), ptr(self.tables[r]), ptr(self.lens[r:]), self.max_blocks,
                                  ptr(self.draft_tables[r]), ptr(self.draft_lens[r:]), self.max_blocks,
                                  ptr(self.free_list), ptr(self.free_top), ptr(self.ref_counts_dev),
                                  self.num_blocks, ptr(rel), 1), "ssd_page_free")
        self._sync_seq(seq, r)
        self._rows.pop(seq.seq_id, None)

    # ------------------------------------------------ batched, sync-free calls
    def allocate_rows(self, row0: int, n: int, num_tokens: torch.Tensor, num_new: torch.Tensor,
                      ok: torch.Tensor | None = None, draft: bool = False) -> None:
        tables = self.draft_tables if draft else self.tables
        lens = self.draft_lens if draft else self.lens
        check(lib().ssd_page_allocate(stream_ptr(), ptr(tables[row0]), ptr(lens[row0:]), self.max_blocks,
                                      ptr(self.free_list), ptr(self.free_top), ptr(self.ref_counts_dev),
                                      self.num_blocks, ptr(num_tokens), ptr(num_new), ptr(ok), self.block_size, n),
              "ssd_page_allocate")

    def rollback_rows(self, row0: int, n: int, num_tokens: torch.Tensor, accepted: torch.Tensor,
                      kv_lens: torch.Tensor | None = None, draft: bool = False) -> None:
        tables = self.draft_tables if draft else self.tables
        lens = self.draft_lens if draft else self.lens
        check(lib().ssd_page_rollback(stream_ptr(), ptr(tables[row0]), ptr(lens[row0:]), self.max_blocks,
                                      ptr(self.free_list), ptr(self.free_top), ptr(self.ref_counts_dev),
                                      self.num_blocks, ptr(num_tokens), ptr(accepted), ptr(kv_lens),
                                      self.block_size, n), "ssd_page_rollback")

    def fork_rows(self, src_row: int, dst_row0: int, n: int, num_tokens: int, cache=None) -> torch.Tensor:
        """Rows dst_row0.. (empty) take src_row's first num_tokens tokens: full blocks shared,
        the partial block copied (K/V rows too when ``cache`` -- a ``KVCacheState`` -- is given).
        Returns ok [n] uint8 (device)."""
        ok = torch.zeros(max(n, 1), dtype=torch.uint8, device=self.device)
        kv, dt, nl, hkv, hd = None, 0, 0, 0, 0
        if cache is not None:
            p = cache.pages
            kv = ptr(p)
            dt = 0 if p.dtype == torch.bfloat16 else 1
            nl, hkv, hd = p.shape[1], p.shape[4], p.shape[5]
        check(lib().ssd_page_fork(stream_ptr(), ptr(self.tables), ptr(self.lens), self.max_blocks,
                                  ptr(self.free_list), ptr(self.free_top), ptr(self.ref_counts_dev), self.num_blocks,
                                  src_row, dst_row0, n, int(num_tokens), self.block_size, ptr(ok), kv, dt, nl, hkv,
                                  hd), "ssd_page_fork")
        return ok[:n]

    def free_rows(self, row0: int, n: int) -> None:
        """Release rows row0 .. row0+n-1 (their blocks' ref counts drop; freed blocks return)."""
        rel = torch.zeros(self.max_seqs, dtype=torch.uint8, device=self.device)
        rel[row0:row0 + n] = 1
        check(lib().ssd_page_free(stream_ptr(), ptr(self.tables), ptr(self.lens), self.max_blocks, None, None, 0,
                                  ptr(self.free_list), ptr(self.free_top), ptr(self.ref_counts_dev),
                                  self.num_blocks, ptr(rel), self.max_seqs), "ssd_page_free")

    def release(self, seq: Sequence) -> None:
        """Forget the slot of a sequence without freeing its blocks (``free_sequence`` does both)."""
        self._rows.pop(seq.seq_id, None)
