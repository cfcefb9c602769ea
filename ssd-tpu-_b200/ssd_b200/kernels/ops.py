"""Thin wrappers over the fused forward ops of libssdverify.so (projections, norms, RoPE)."""

from __future__ import annotations

import torch

from .._lib import (SSD_EPI_GEGLU, SSD_EPI_RESIDUAL, SSD_EPI_STORE, SSD_EPI_STORE_F32, check, dtype_code,
                    lib, ptr, stream_ptr)
from ..workspace import workspace

EPILOGUES = {"store": SSD_EPI_STORE, "store_f32": SSD_EPI_STORE_F32, "residual": SSD_EPI_RESIDUAL,
             "geglu": SSD_EPI_GEGLU}


def linear(x: torch.Tensor, w: torch.Tensor, epilogue: str = "store", out: torch.Tensor | None = None,
           ws_key: str = "linear", rownorm_eps: float | None = None) -> torch.Tensor:
    """epilogue(x[M,K] w[N,K]^T); ``residual`` accumulates into ``out`` in place.

    With ``rownorm_eps`` the result rows are scaled by rsqrt(mean(x^2) + eps)
    (``ssd_linear_rownorm``: an RMSNorm whose weight is folded into ``w``).
    """
    m, k = x.shape
    n = w.shape[0]
    epi = EPILOGUES[epilogue]
    if out is None:
        if epi == SSD_EPI_RESIDUAL:
            raise ValueError("residual epilogue needs out=")
        cols = n // 2 if epi == SSD_EPI_GEGLU else n
        out = torch.empty((m, cols), dtype=torch.float32 if epi == SSD_EPI_STORE_F32 else x.dtype, device=x.device)
    ws = workspace(x.device, ws_key, lib().ssd_linear_workspace_size(m, n, k))
    if rownorm_eps is not None:
        check(lib().ssd_linear_rownorm(stream_ptr(), ptr(x), ptr(w), dtype_code(w.dtype), ptr(out), epi, m, n, k,
                                       float(rownorm_eps), ptr(ws), ws.numel()), "ssd_linear_rownorm")
        return out
    check(lib().ssd_linear(stream_ptr(), ptr(x), ptr(w), dtype_code(w.dtype), ptr(out), epi, m, n, k, ptr(ws),
                           ws.numel()), "ssd_linear")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    m, d = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().ssd_rmsnorm(stream_ptr(), ptr(x), ptr(w), dtype_code(x.dtype), ptr(out), m, d, float(eps)),
          "ssd_rmsnorm")
    return out


def embed(tokens: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    m = tokens.numel()
    v, d = table.shape
    out = torch.empty((m, d), dtype=table.dtype, device=table.device) if out is None else out
    check(lib().ssd_embed(stream_ptr(), ptr(tokens), ptr(table), dtype_code(table.dtype), ptr(out), m, d, v),
          "ssd_embed")
    return out


def max_tokens_per_forward(dtype=None) -> int:
    """Largest B*T one forward takes: 256 on the tcgen05 (bf16) path, 16 on the fp32 CUDA-core path."""
    import torch

    if dtype == torch.float32:
        return 16
    return int(lib().ssd_linear_max_m())


def linear_allreduce(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, comm, ws_key: str = "linear") -> torch.Tensor:
    """y[M,N] += sum over the tensor-parallel ranks of x_r w_r^T (bf16; ``ssd_linear_allreduce``)."""
    import ctypes as C

    m, k = x.shape
    n = w.shape[0]
    nbytes = lib().ssd_linear_workspace_size(m, n, k)
    ws = workspace(x.device, ws_key, nbytes)
    check(lib().ssd_linear_allreduce(stream_ptr(), ptr(x), ptr(w), ptr(y), m, n, k, ptr(ws), ws.numel(),
                                     C.byref(comm.cstruct)), "ssd_linear_allreduce")
    return y


def linear_allgather(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, comm, ws_key: str = "linear") -> torch.Tensor:
    """y[M, rank*N:(rank+1)*N] = x w^T (fp32) on every rank; y from ``comm.alloc`` (``ssd_linear_allgather``)."""
    import ctypes as C

    m, k = x.shape
    n = w.shape[0]
    nbytes = lib().ssd_linear_workspace_size(m, n, k)
    ws = workspace(x.device, ws_key, nbytes)
    check(lib().ssd_linear_allgather(stream_ptr(), ptr(x), ptr(w), ptr(y), y.shape[-1], m, n, k, ptr(ws),
                                     ws.numel(), C.byref(comm.cstruct)), "ssd_linear_allgather")
    return y
