"""Runtime configuration (same fields as jax_ssd/config.py:40-68).

Model "paths" name random-init presets of ``models.gemma.PRESETS`` ("gemma-7b",
"gemma-2b", "toy-target", "toy-draft"): there are no checkpoints in this
build's benchmarks.  ``use_toy_model`` (env ``SSD_USE_TOY_MODEL``) selects the
Gemma-style toy pair of the benchmark's CPU parity config.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from enum import Enum


def _env_bool(key: str, default: bool = False) -> bool:
    return os.getenv(key, "1" if default else "0").lower() in ("1", "true", "yes")


class DecodeMode(str, Enum):
    AR = "ar"
    SD = "sd"
    SSD = "ssd"
    INSTANCE = "instance"


@dataclass
class SSDConfig:
    mode: DecodeMode = DecodeMode.AR
    speculate_k: int = 4
    fan_out_list: tuple[int, ...] = (2, 2, 2, 2, 2)
    sampler_x: float = 0.5
    max_model_len: int = 4096
    block_size: int = 16
    num_blocks: int = 256
    batch_buckets: tuple[int, ...] = (1, 2, 4, 8, 16)
    target_model_path: str | None = field(default_factory=lambda: os.getenv("TARGET_MODEL_PATH"))
    draft_model_path: str | None = field(default_factory=lambda: os.getenv("DRAFT_MODEL_PATH"))
    use_toy_model: bool = field(default_factory=lambda: _env_bool("SSD_USE_TOY_MODEL"))
    # ssd mode: the draft model and its worker on their own GPU (e.g. "cuda:1"); None = the next GPU after
    # the target's tensor-parallel group when there is one, else the target's GPU
    draft_device: str | None = field(default_factory=lambda: os.getenv("SSD_DRAFT_DEVICE"))
    # target tensor parallelism over GPUs 0..tensor_parallel_size-1 (one process, one thread per GPU);
    # in sd and ar modes the draft is sharded over the same GPUs, in ssd mode it runs on draft_device
    tensor_parallel_size: int = field(default_factory=lambda: int(os.getenv("SSD_TP_SIZE", "1")))
    tpu_role: str = field(default_factory=lambda: os.getenv("SSD_TPU_ROLE", "both").lower())
    mesh_allocation: object | None = None
    instance_context_ratio: float = 0.3
    seed: int = 0

    @property
    def mq_len(self) -> int:
        k = self.speculate_k
        fan = self.fan_out_list
        if len(fan) < k + 1:
            fan = fan + (fan[-1],) * (k + 1 - len(fan))
        return sum(fan[: k + 1])

    @classmethod
    def from_fanout_string(cls, fanout: str, **kwargs) -> "SSDConfig":
        fl = tuple(int(x.strip()) for x in fanout.split(",") if x.strip())
        return cls(fan_out_list=fl, **kwargs)
