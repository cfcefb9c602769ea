"""Run metrics of the engine.

The record types keep the reference's field names (``StepMetrics`` and
``RunMetrics`` of jax_ssd/runtime/metrics.py:10-51: tokens/s, TTFT, cache hit
rate, ``to_dict``) so that callers reading them switch modules only.  The
recording side is this engine's own: a ``MetricsCollector`` is a timeline of
monotonic-clock marks plus running totals, filled per engine step (one step
may emit tokens for many sequences at once in the batched engine), and it also
keeps what the device path measures -- CUDA-event verify time per step and the
distribution of accepted draft counts.
"""

from __future__ import annotations

import time
from collections import Counter
from dataclasses import dataclass, field


@dataclass
class StepMetrics:
    """One engine step: wall time of the step, tokens it emitted, whether the draft came from the cache."""

    target_verify_ms: float = 0.0  # host wall time of the step (draft + verify + commit)
    draft_step_ms: float = 0.0
    cache_hit: bool = False
    accepted_tokens: int = 0       # tokens emitted by the step (accepted drafts + recovery/bonus, all sequences)
    verify_device_ms: float = 0.0  # CUDA-event time of the target forward + acceptance
    sequences: int = 1             # sequences the step advanced


@dataclass
class RunMetrics:
    mode: str = "ar"
    total_tokens: int = 0
    total_time_s: float = 0.0
    ttft_s: float = 0.0
    cache_hits: int = 0
    cache_misses: int = 0
    steps: list[StepMetrics] = field(default_factory=list)
    accept_histogram: dict[int, int] = field(default_factory=dict)  # accepted drafts per sequence-step -> count

    @property
    def tokens_per_second(self) -> float:
        return self.total_tokens / self.total_time_s if self.total_time_s > 0 else 0.0

    @property
    def cache_hit_rate(self) -> float:
        n = self.cache_hits + self.cache_misses
        return self.cache_hits / n if n else 0.0

    @property
    def accepted_per_step(self) -> float:
        """Mean tokens one sequence gains per verify step (accepted drafts + the recovery/bonus token)."""
        seq_steps = sum(s.sequences for s in self.steps)
        return self.total_tokens / seq_steps if seq_steps else 0.0

    @property
    def verify_device_ms(self) -> float:
        """Mean CUDA-event time of the verify forward + acceptance over the steps that recorded one."""
        timed = [s.verify_device_ms for s in self.steps if s.verify_device_ms > 0]
        return sum(timed) / len(timed) if timed else 0.0

    def to_dict(self) -> dict:
        keys = ("mode", "total_tokens", "total_time_s", "tokens_per_second", "ttft_s", "cache_hit_rate",
                "cache_hits", "cache_misses", "accepted_per_step", "verify_device_ms")
        out = {k: getattr(self, k) for k in keys}
        out["num_steps"] = len(self.steps)
        out["accept_histogram"] = dict(sorted(self.accept_histogram.items()))
        return out


class MetricsCollector:
    """Timeline of one ``generate`` call.

    ``start`` opens it; ``record_first_token`` marks the first emitted token
    (TTFT, once); ``record_step`` appends a step and updates the totals;
    ``record_accepts`` adds per-sequence accepted-draft counts to the histogram;
    ``finish`` closes the timeline and returns the ``RunMetrics``.
    """

    def __init__(self, mode: str) -> None:
        self._mode = mode
        self._marks: dict[str, int] = {}
        self._steps: list[StepMetrics] = []
        self._tokens = 0
        self._hits = Counter()
        self._accepts = Counter()

    def _mark(self, name: str) -> None:
        self._marks.setdefault(name, time.monotonic_ns())

    def start(self) -> None:
        self._marks.clear()
        self._mark("start")

    def record_first_token(self) -> None:
        if "start" in self._marks:
            self._mark("first_token")

    def record_step(self, step: StepMetrics) -> None:
        self._steps.append(step)
        self._tokens += step.accepted_tokens
        self._hits[bool(step.cache_hit)] += 1

    def record_accepts(self, accepted) -> None:
        for a in accepted:
            self._accepts[int(a)] += 1

    def finish(self) -> RunMetrics:
        self._mark("end")
        t0 = self._marks.get("start")
        elapsed = lambda name: (self._marks[name] - t0) / 1e9 if t0 is not None and name in self._marks else 0.0  # noqa: E731
        return RunMetrics(mode=self._mode, total_tokens=self._tokens, total_time_s=elapsed("end"),
                          ttft_s=elapsed("first_token"), cache_hits=self._hits[True],
                          cache_misses=self._hits[False], steps=list(self._steps),
                          accept_histogram=dict(self._accepts))

    @property
    def metrics(self) -> RunMetrics:
        """The run so far (the timeline stays open)."""
        t0 = self._marks.get("start")
        now = time.monotonic_ns()
        return RunMetrics(mode=self._mode, total_tokens=self._tokens,
                          total_time_s=(now - t0) / 1e9 if t0 is not None else 0.0,
                          ttft_s=(self._marks["first_token"] - t0) / 1e9 if "first_token" in self._marks else 0.0,
                          cache_hits=self._hits[True], cache_misses=self._hits[False], steps=list(self._steps),
                          accept_histogram=dict(self._accepts))
