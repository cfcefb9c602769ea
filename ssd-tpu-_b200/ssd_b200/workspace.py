"""Caller-owned device workspaces for the C ABI (which never allocates).

Each buffer is zero-filled when allocated; the kernels leave their workspace
zero-filled again after every call, so buffers are reused without a memset.
Buffers are keyed by purpose so calls that may overlap never share one.
"""

from __future__ import annotations

import torch

_POOLS: dict[tuple[int, str], torch.Tensor] = {}


def workspace(device: torch.device | int, key: str, nbytes: int) -> torch.Tensor:
    dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    k = (idx, key)
    buf = _POOLS.get(k)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=torch.device("cuda", idx))
        _POOLS[k] = buf
    return buf


def release_all() -> None:
    _POOLS.clear()
