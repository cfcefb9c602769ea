"""Speculative-decoding acceptance on the GPU (drop-in for jax_ssd/algorithm/verify.py).

``verify_greedy`` and ``verify_sample`` keep the reference signatures
(``jax_ssd/algorithm/verify.py:18-23,68-77``) and return the same
``VerifyResult`` fields (:11-15); the work runs in the fused K4 kernels of
``libssdverify.so`` (``ssd_verify_greedy`` / ``ssd_verify_sample``).

Random draws: the reference consumes a JAX PRNG key through
``jax.random.split/uniform/categorical`` (verify.py:80,100,107,113,119), which
cannot be reproduced outside JAX.  Here ``key`` is either an ``int`` seed —
expanded on the device by the counter-based ``ssd_uniform_fill`` into
``u_accept[B,K]`` and ``u_gumbel[B,V]`` — or an explicit ``(u_accept, u_gumbel)``
pair, which is how parity tests feed both sides identical draws.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib
from .._lib import check, lib, ptr, stream_ptr
from ..workspace import workspace


@dataclass(frozen=True)
class VerifyResult:
    accept_until: torch.Tensor     # [B] int32 -- number of draft tokens accepted (0..K)
    recovery_tokens: torch.Tensor  # [B] int32
    accepted_mask: torch.Tensor    # [B, K+1] bool


def _dev(x, dtype) -> torch.Tensor:
    t = torch.as_tensor(x)
    if not t.is_cuda:
        t = t.to("cuda")
    return t.to(dtype).contiguous()


def verify_greedy(logits_p, speculations, *, cache_hit=None, target_tokens: bool = False):
    """verify.py:18-59: greedy acceptance over K+1 positions.

    logits_p [B, K+1, V] fp32, speculations [B, K+1] int32 (column 0 = previous
    recovery token).  ``cache_hit`` is accepted for signature compatibility and,
    as in the reference (:52-53), does not change the greedy result.  With
    ``target_tokens=True`` the per-position argmax [B, K+1] is returned too.
    """
    lp = _dev(logits_p, torch.float32)
    spec = _dev(speculations, torch.int32)
    b, kp1, v = lp.shape
    k = kp1 - 1
    if spec.shape != (b, kp1):
        raise ValueError(f"speculations must be [{b}, {kp1}], got {tuple(spec.shape)}")
    acc = torch.empty(b, dtype=torch.int32, device=lp.device)
    rec = torch.empty(b, dtype=torch.int32, device=lp.device)
    mask = torch.empty((b, kp1), dtype=torch.uint8, device=lp.device)
    tt = torch.empty((b, kp1), dtype=torch.int32, device=lp.device) if target_tokens else None
    nbytes = lib().ssd_verify_greedy_workspace_size(b, k, v)
    ws = workspace(lp.device, "verify_greedy", nbytes)
    check(lib().ssd_verify_greedy(stream_ptr(), ptr(lp), ptr(spec), ptr(acc), ptr(rec), ptr(mask), ptr(tt),
                                  ptr(ws), ws.numel(), b, k, v), "ssd_verify_greedy")
    res = VerifyResult(acc, rec, mask.view(torch.bool))
    return (res, tt) if target_tokens else res


def uniforms_from_seed(seed: int, b: int, k: int, v: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Counter-based (0,1) draws: u_accept = stream[0 : B*K], u_gumbel = stream[B*K : B*K + B*V]."""
    ua = torch.empty((b, k), dtype=torch.float32, device=device)
    ug = torch.empty((b, v), dtype=torch.float32, device=device)
    check(lib().ssd_uniform_fill(stream_ptr(), ptr(ua), ua.numel(), seed & (2**64 - 1), 0), "ssd_uniform_fill")
    check(lib().ssd_uniform_fill(stream_ptr(), ptr(ug), ug.numel(), seed & (2**64 - 1), b * k), "ssd_uniform_fill")
    return ua, ug


def top_p_mask_(x: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """In place: every logit of each row of ``x`` below the top-p cutoff of softmax(x / temperature)
    becomes -inf (``ssd_top_p_mask``; ties at the cutoff are kept, NaN is masked).  ``x`` is a 2-D
    (or [..., V] contiguous) fp32 CUDA tensor; top_p >= 1 leaves it untouched."""
    if x.dtype != torch.float32 or not x.is_cuda or x.stride(-1) != 1:
        raise ValueError("top_p_mask_ wants a row-contiguous fp32 CUDA tensor")
    v = x.shape[-1]
    rows = x.numel() // v if x.dim() != 2 else x.shape[0]
    ld = x.stride(0) if x.dim() == 2 else v
    if x.dim() != 2 and not x.is_contiguous():
        raise ValueError("top_p_mask_ wants a contiguous tensor when it is not 2-D")
    check(lib().ssd_top_p_mask(stream_ptr(), ptr(x), ld, rows, v, float(temperature), float(top_p)),
          "ssd_top_p_mask")
    return x


def verify_sample(logits_p, logits_q, speculations, key, *, temperature_p: float = 1.0,
                  temperature_q: float = 1.0, sampler_x: float = 0.5, alignment: str = "reference",
                  top_p: float = 1.0):
    """verify.py:68-120: rejection sampling with bonus token and residual draw.

    logits_p [B, K+1, V], logits_q [B, K, V] fp32; speculations [B, K+1].
    ``key``: int seed or ``(u_accept[B,K], u_gumbel[B,V])``.
    ``alignment="reference"`` judges draft token j+1 with target row j+1, as
    verify.py:103 does; ``"standard"`` uses row j (the textbook rule).
    ``top_p < 1`` (not in the reference) runs the test on the top-p nuclei of
    both distributions (``top_p_mask_`` on copies of the logits).
    """
    lp = _dev(logits_p, torch.float32)
    lq = _dev(logits_q, torch.float32)
    if top_p < 1.0:
        lp = top_p_mask_(lp.clone(), temperature_p, top_p)
        lq = top_p_mask_(lq.clone(), temperature_q, top_p) if lq.numel() else lq
    spec = _dev(speculations, torch.int32)
    b, kp1, v = lp.shape
    k = kp1 - 1
    if lq.shape != (b, k, v) or spec.shape != (b, kp1):
        raise ValueError("shape mismatch between logits_p, logits_q and speculations")
    if isinstance(key, (tuple, list)):
        ua, ug = _dev(key[0], torch.float32), _dev(key[1], torch.float32)
    else:
        ua, ug = uniforms_from_seed(int(key), b, k, v, lp.device)
    if temperature_p <= 0 or temperature_q <= 0:
        raise ValueError("sampling temperatures must be > 0 (use verify_greedy for temperature 0)")
    align = _lib.SSD_ALIGN_REFERENCE if alignment == "reference" else _lib.SSD_ALIGN_STANDARD
    acc = torch.empty(b, dtype=torch.int32, device=lp.device)
    rec = torch.empty(b, dtype=torch.int32, device=lp.device)
    mask = torch.empty((b, kp1), dtype=torch.uint8, device=lp.device)
    nbytes = lib().ssd_verify_sample_workspace_size(b, k, v)
    ws = workspace(lp.device, "verify_sample", nbytes)
    check(lib().ssd_verify_sample(stream_ptr(), ptr(lp), ptr(lq), ptr(spec), ptr(ua), ptr(ug),
                                  float(temperature_p), float(temperature_q), float(sampler_x), align,
                                  ptr(acc), ptr(rec), ptr(mask), ptr(ws), ws.numel(), b, k, v),
          "ssd_verify_sample")
    return VerifyResult(acc, rec, mask.view(torch.bool))


def argmax_rows(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """First-index argmax of each row of a 2-D fp32 CUDA tensor (ssd_argmax_rows)."""
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
        raise ValueError("argmax_rows wants a row-contiguous 2-D fp32 CUDA tensor")
    rows, v = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    nbytes = lib().ssd_verify_greedy_workspace_size(rows, 0, v)
    ws = workspace(x.device, "argmax_rows", nbytes)
    check(lib().ssd_argmax_rows(stream_ptr(), ptr(x), x.stride(0), rows, v, ptr(out), ptr(ws), ws.numel()),
          "ssd_argmax_rows")
    return out


def sample_rows(x: torch.Tensor, temperature: float, seed: int, offset: int = 0,
                out: torch.Tensor | None = None, top_p: float = 1.0) -> torch.Tensor:
    """One draw per row from softmax(x / temperature) (``ssd_sample_rows``, Gumbel-max on a counter hash).

    The draw for (seed, offset) is reproducible; callers advance ``offset`` by at
    least rows * V between draws that must be independent.  ``top_p < 1`` draws
    from the top-p nucleus (``top_p_mask_`` on a copy of ``x``).
    """
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
        raise ValueError("sample_rows wants a row-contiguous 2-D fp32 CUDA tensor")
    if top_p < 1.0:
        x = top_p_mask_(x.clone(), temperature, top_p)
    rows, v = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    nbytes = lib().ssd_verify_greedy_workspace_size(rows, 0, v)
    ws = workspace(x.device, "sample_rows", nbytes)
    check(lib().ssd_sample_rows(stream_ptr(), ptr(x), x.stride(0), rows, v, float(temperature),
                                int(seed) & (2**64 - 1), int(offset) & (2**64 - 1), ptr(out), ptr(ws), ws.numel()),
          "ssd_sample_rows")
    return out
