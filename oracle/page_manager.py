"""Oracle: paged-KV block allocation and speculative rollback (test infrastructure only).

Restates ``jax_ssd/runtime/page_manager.py`` of the reference:

* ``allocate`` / ``allocate_draft`` — page_manager.py:21-33 / :35-47.  Blocks are
  popped from the END of the free list (LIFO, :30) and appended to the table.
  If fewer free blocks remain than needed, nothing changes and False returns.
* ``rollback_speculative`` — page_manager.py:49-56.  ``used =
  ceil((num_tokens + accepted) / block_size)``; blocks are popped from the end
  of the table while ``len > used`` (the second clause of :53 reduces to
  ``len > used`` as well, so ``reserved`` has no effect).
* ``free_sequence`` — page_manager.py:58-64: the target table in forward order,
  then the draft table.
* ``_free_block`` — page_manager.py:66-70: ``rc = ref_counts.get(b, 1) - 1``; at
  ``rc <= 0`` the entry is deleted and the block is appended to the free list.

The dense form used by the device kernels stores the dict as an int32 array
(0 = absent) and the free list as a stack ``free_list[:free_top]``; per-event
release is then ``rc' = max(rc, 1) - 1`` with a push when ``rc' == 0``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class OracleSeq:
    """jax_ssd/runtime/sequence.py:16-36 (only the fields the allocator reads)."""

    num_tokens: int
    block_table: list = field(default_factory=list)
    draft_block_table: list = field(default_factory=list)


@dataclass
class OraclePageManager:
    block_size: int
    num_blocks: int
    free_blocks: list = field(default_factory=list)
    ref_counts: dict = field(default_factory=dict)

    def __post_init__(self):
        if not self.free_blocks:
            self.free_blocks = list(range(self.num_blocks))

    def _alloc(self, table: list, num_tokens_now: int, n: int) -> bool:
        need = (num_tokens_now + n + self.block_size - 1) // self.block_size
        extra = need - len(table)
        if extra <= 0:
            return True
        if len(self.free_blocks) < extra:
            return False
        for _ in range(extra):
            blk = self.free_blocks.pop()
            table.append(blk)
            self.ref_counts[blk] = self.ref_counts.get(blk, 0) + 1
        return True

    def allocate(self, seq: OracleSeq, n: int) -> bool:
        return self._alloc(seq.block_table, seq.num_tokens, n)

    def allocate_draft(self, seq: OracleSeq, n: int) -> bool:
        return self._alloc(seq.draft_block_table, seq.num_tokens, n)

    def rollback_speculative(self, seq: OracleSeq, accepted: int, reserved: int) -> None:
        used = (seq.num_tokens + accepted + self.block_size - 1) // self.block_size
        while len(seq.block_table) > used:
            self._free_block(seq.block_table.pop())

    def free_sequence(self, seq: OracleSeq) -> None:
        for blk in seq.block_table:
            self._free_block(blk)
        for blk in seq.draft_block_table:
            self._free_block(blk)
        seq.block_table.clear()
        seq.draft_block_table.clear()

    def fork(self, src: OracleSeq, dsts: list, num_tokens: int) -> list:
        """Branch fork (no reference counterpart; the device ``ssd_page_fork``): each empty
        dst takes src's first num_tokens tokens -- full blocks shared with ref counts
        ``get(b, 1) + 1`` (the reading of page_manager.py:66-70), a fresh LIFO-popped block
        for a partial last block.  Returns ok per dst (False: left empty, nothing popped)."""
        full, part = divmod(num_tokens, self.block_size)
        need = full + (1 if part else 0)
        oks = []
        for d in dsts:
            fits = len(src.block_table) >= need and (not part or len(self.free_blocks) > 0)
            oks.append(fits)
            if not fits:
                continue
            d.block_table = list(src.block_table[:full])
            for blk in d.block_table:
                self.ref_counts[blk] = self.ref_counts.get(blk, 1) + 1
            if part:
                blk = self.free_blocks.pop()
                d.block_table.append(blk)
                self.ref_counts[blk] = self.ref_counts.get(blk, 0) + 1
        return oks

    def _free_block(self, blk: int) -> None:
        rc = self.ref_counts.get(blk, 1) - 1
        self.ref_counts[blk] = rc
        if rc <= 0:
            del self.ref_counts[blk]
            self.free_blocks.append(blk)


# ---------------------------------------------------------------- dense form
def to_dense(pm: OraclePageManager, seqs: list, max_blocks: int):
    """List state -> (tables[S,M], lens[S], free_list[NB], free_top, ref_counts[NB])."""
    s = len(seqs)
    tables = np.full((s, max_blocks), -1, np.int32)
    lens = np.zeros(s, np.int32)
    for i, q in enumerate(seqs):
        tables[i, : len(q.block_table)] = q.block_table
        lens[i] = len(q.block_table)
    free = np.full(pm.num_blocks, -1, np.int32)
    free[: len(pm.free_blocks)] = pm.free_blocks
    rc = np.zeros(pm.num_blocks, np.int32)
    for kk, vv in pm.ref_counts.items():
        rc[int(kk)] = vv
    return tables, lens, free, np.int32(len(pm.free_blocks)), rc


def dense_rollback(tables, lens, free, free_top, rc, num_tokens, accepted, block_size):
    """Batched rollback in sequence order (seq 0 first), dense form, as the kernel does it."""
    tables, lens, free, rc = tables.copy(), lens.copy(), free.copy(), rc.copy()
    top = int(free_top)
    for i in range(tables.shape[0]):
        used = (int(num_tokens[i]) + int(accepted[i]) + block_size - 1) // block_size
        while lens[i] > used:
            lens[i] -= 1
            blk = int(tables[i, lens[i]])
            tables[i, lens[i]] = -1
            nv = max(int(rc[blk]), 1) - 1
            rc[blk] = nv
            if nv == 0:
                free[top] = blk
                top += 1
    return tables, lens, free, np.int32(top), rc


def dense_allocate(tables, lens, free, free_top, rc, num_tokens, n_new, block_size):
    """Batched allocate in sequence order; returns the new state and ok[S] (bool)."""
    tables, lens, free, rc = tables.copy(), lens.copy(), free.copy(), rc.copy()
    top = int(free_top)
    ok = np.ones(tables.shape[0], bool)
    for i in range(tables.shape[0]):
        need = (int(num_tokens[i]) + int(n_new[i]) + block_size - 1) // block_size
        extra = need - int(lens[i])
        if extra <= 0:
            continue
        if top < extra or lens[i] + extra > tables.shape[1]:
            ok[i] = False
            continue
        for _ in range(extra):
            top -= 1
            blk = int(free[top])
            free[top] = -1
            tables[i, lens[i]] = blk
            lens[i] += 1
            rc[blk] += 1
    return tables, lens, free, np.int32(top), rc, ok
