"""Slot scheduler for the batched serving loop.

The reference's scheduler (jax_ssd/runtime/scheduler.py:12-77) keeps a
waiting deque and a running list and reserves KV pages on the host that its
model never reads; its engine then decodes one prompt at a time
(jax_ssd/runtime/engine.py:110-125).  Here the KV pages live on the device with
each decoder (``PageManager`` rows), and one decoder step advances a fixed set
of B rows together.  This scheduler's job is the mapping between requests and
those rows ("slots"):

* ``add_request`` queues a prompt as a ``Sequence`` (WAITING);
* ``admit`` places waiting sequences into free slots, first come first served,
  and returns the (slot, sequence) pairs the decoder must prefill;
* ``retire`` frees a slot whose sequence has finished, so the next ``admit``
  refills it while the other rows keep decoding (continuous batching);
* ``slots`` lists the occupied slots in slot order.

A slot with no sequence still steps inside the decoder (its rows are part of
the fixed-shape batch); the engine parks it on a one-token dummy sequence and
ignores what it produces.
"""

from __future__ import annotations

from collections import deque

from .sequence import Sequence, SequenceStatus


class Scheduler:
    def __init__(self, num_slots: int) -> None:
        if num_slots < 1:
            raise ValueError("the scheduler needs at least one slot")
        self.num_slots = int(num_slots)
        self.waiting: deque[Sequence] = deque()
        self.finished: list[Sequence] = []
        self._slot_seq: list[Sequence | None] = [None] * self.num_slots
        self._ids = 0

    # ------------------------------------------------------------ queue
    def add_request(self, prompt_token_ids: list[int]) -> Sequence:
        seq = Sequence(seq_id=self._ids, prompt_token_ids=[int(t) for t in prompt_token_ids])
        self._ids += 1
        self.waiting.append(seq)
        return seq

    def has_work(self) -> bool:
        return bool(self.waiting) or any(s is not None for s in self._slot_seq)

    # ------------------------------------------------------------ slots
    @property
    def running(self) -> list[Sequence]:
        return [s for s in self._slot_seq if s is not None]

    def slots(self) -> list[tuple[int, Sequence]]:
        return [(i, s) for i, s in enumerate(self._slot_seq) if s is not None]

    def free_slots(self) -> list[int]:
        return [i for i, s in enumerate(self._slot_seq) if s is None]

    def admit(self) -> list[tuple[int, Sequence]]:
        placed = []
        for slot in self.free_slots():
            if not self.waiting:
                break
            seq = self.waiting.popleft()
            seq.status = SequenceStatus.RUNNING
            self._slot_seq[slot] = seq
            placed.append((slot, seq))
        return placed

    def retire(self, slot: int) -> Sequence:
        seq = self._slot_seq[slot]
        if seq is None:
            raise ValueError(f"slot {slot} holds no sequence")
        seq.status = SequenceStatus.FINISHED
        self._slot_seq[slot] = None
        self.finished.append(seq)
        return seq
