"""Generation controls (jax_ssd/sampling_params.py:8-13, plus ``top_p``)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SamplingParams:
    temperature: float = 0.0
    draft_temperature: float = 0.0
    max_new_tokens: int = 128
    ignore_eos: bool = False
    # not in the reference: nucleus filtering of the target and draft distributions when temperature > 0
    top_p: float = 1.0
