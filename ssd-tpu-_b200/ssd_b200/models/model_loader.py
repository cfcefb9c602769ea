"""Load target/draft adapters (jax_ssd/models/model_loader.py:40-76).

There are no checkpoints here: a model "path" names a random-init preset of
``models.gemma.PRESETS`` (default: "gemma-7b" target, "gemma-2b" draft; the toy
pair with ``use_toy``).  Weights are initialised on the device from the seed.
"""

from __future__ import annotations

import os

import torch

from .gemma import PRESETS, GemmaWeights
from .gemma_adapter import GemmaAdapter

_SHARED: dict[tuple, GemmaWeights] = {}


def default_target_path() -> str:
    """TARGET_MODEL_PATH, else the Gemma-7B preset (model_loader.py:26-30 defaults to a checkpoint URL)."""
    return os.getenv("TARGET_MODEL_PATH", "gemma-7b")


def default_draft_path() -> str:
    """DRAFT_MODEL_PATH, else the Gemma-2B preset (model_loader.py:33-37)."""
    return os.getenv("DRAFT_MODEL_PATH", "gemma-2b")


def default_preset(role: str, use_toy: bool) -> str:
    if use_toy:
        return "toy-target" if role == "target" else "toy-draft"
    return "gemma-7b" if role == "target" else "gemma-2b"


def load_weights(model_path: str | None, *, use_toy: bool = False, seed: int = 0, role: str = "target",
                 device="cuda") -> GemmaWeights:
    name = model_path if model_path in PRESETS else default_preset(role, use_toy)
    dtype = torch.float32 if name.startswith("toy") else torch.bfloat16
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (name, seed, str(dev))
    w = _SHARED.get(key)
    if w is None:
        with torch.cuda.device(dev):  # the init kernels run on that GPU's current stream
            w = GemmaWeights.random(PRESETS[name], seed=seed, dtype=dtype, device=dev)
            torch.cuda.current_stream(dev).synchronize()
        _SHARED[key] = w
    return w


def load_sharded_weights(model_path: str | None, rank: int, world: int, *, use_toy: bool = False, seed: int = 0,
                         role: str = "target", device="cuda") -> GemmaWeights:
    """Rank ``rank``'s tensor-parallel shard (``runtime.tensor_parallel.shard_weights``) of the
    weights ``load_weights`` would give: the full model is drawn from the seed on ``device``, sharded,
    and dropped, so every rank holds the same model's shard."""
    from ..runtime.tensor_parallel import shard_weights

    name = model_path if model_path in PRESETS else default_preset(role, use_toy)
    if name.startswith("toy"):
        raise ValueError("tensor parallelism runs on bf16 weights; the fp32 toy pair has no sharded path "
                         "(the tp-target / tp-draft presets are small bf16 models)")
    dev = torch.device(device)
    key = (name, seed, str(dev), rank, world)
    w = _SHARED.get(key)
    if w is None:
        with torch.cuda.device(dev):
            full = GemmaWeights.random(PRESETS[name], seed=seed, dtype=torch.bfloat16, device=dev)
            w = shard_weights(full, rank, world)
            torch.cuda.current_stream(dev).synchronize()
            del full
            torch.cuda.empty_cache()
        _SHARED[key] = w
    return w


def load_model_adapter(model_path: str | None, *, use_toy: bool = False, seed: int = 0, share_key=None,
                       mesh=None, devices=None, role: str = "target", max_model_len: int = 4096) -> GemmaAdapter:
    w = load_weights(model_path, use_toy=use_toy, seed=seed, role=role)
    return GemmaAdapter(w, max_model_len=max_model_len, name=role)
