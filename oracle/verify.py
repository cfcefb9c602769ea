"""Oracle: greedy and sampling-mode acceptance (test infrastructure only).

Restates ``jax_ssd/algorithm/verify.py`` of the reference:

* ``verify_greedy``  — verify.py:18-59
* ``softmax``        — verify.py:62-65
* ``verify_sample``  — verify.py:68-120, with the reference's JAX threefry
  draws replaced by explicit uniform arrays: ``u_accept[B, K]`` for the
  accept tests (``jax.random.uniform(keys[j])``, :107) and ``u_gumbel[B, V]``
  for the final categorical draw (``jax.random.categorical(keys[k+1], ...)``,
  :113/:119), which JAX computes as ``argmax(logits - log(-log(u)))``.

Alignment: the reference's ``_verify_sample_row`` judges draft token
``spec[j+1]`` with target row ``lp[j+1]`` (:103) while ``verify_greedy`` uses
``lp[j]`` (:35-36).  ``alignment="reference"`` reproduces the former as
written; ``alignment="standard"`` uses ``lp[j]`` (and ``lp[acc]`` for the
residual), which is the textbook rule.
"""

from __future__ import annotations

import numpy as np


def verify_greedy(logits_p: np.ndarray, speculations: np.ndarray):
    """verify.py:18-59. Returns (accept_until[B], recovery[B], accepted_mask[B,K+1])."""
    b, kp1, _ = logits_p.shape
    k = kp1 - 1
    t = np.argmax(logits_p, axis=-1).astype(np.int32)  # first index on ties
    matches = speculations[:, 1:] == t[:, :k]
    acc = np.cumprod(matches.astype(np.int32), axis=1).sum(axis=1).astype(np.int32)
    rec = np.where(acc == k, t[:, k], t[np.arange(b), np.minimum(acc, k)]).astype(np.int32)
    mask = np.zeros((b, kp1), dtype=bool)
    mask[:, 1:] = np.arange(k)[None, :] < acc[:, None]
    return acc, rec, mask


def softmax(x: np.ndarray) -> np.ndarray:
    """verify.py:62-65 in fp32: exp(x - max) / sum."""
    x = x.astype(np.float32)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def top_p_threshold(x: np.ndarray, temperature: float, top_p: float):
    """Cutoff of the top-p nucleus of softmax(x / T) for one row (fp32 logits).

    Not in the reference (its SamplingParams has no top-p); restates the
    definition ``ssd_top_p_mask`` implements: fp64 masses w = exp(-(m - x) / T)
    over the finite logits, sorted by value (descending); the cutoff is the
    value at which the running mass first reaches top_p * Z, so every logit
    >= it (ties included) is kept.  None: no finite logit.
    """
    v = np.asarray(x, dtype=np.float32)
    fin = v > -np.inf  # False for -inf and NaN
    if not fin.any():
        return None
    vals = v[fin].astype(np.float64)
    m = vals.max()
    inv_t = 1.0 / float(np.float32(temperature))
    w = np.exp(-((m - vals) * inv_t))
    order = np.argsort(-vals, kind="stable")
    cum = np.cumsum(w[order])
    i = int(np.searchsorted(cum, top_p * w.sum(), side="left"))
    if i >= len(vals):
        return np.float32(-np.inf)
    return np.float32(vals[order][i])


def top_p_mask(x: np.ndarray, temperature: float, top_p: float) -> np.ndarray:
    """Copy of logits [..., V] with every value below its row's top-p cutoff (and NaN) set to -inf."""
    out = np.array(x, dtype=np.float32, copy=True)
    if top_p >= 1.0:
        return out
    rows = out.reshape(-1, out.shape[-1])
    for r in rows:
        t = top_p_threshold(r, temperature, top_p)
        if t is None:
            continue
        r[~(r >= t)] = -np.inf
    return out


def verify_sample(
    logits_p: np.ndarray,
    logits_q: np.ndarray,
    speculations: np.ndarray,
    u_accept: np.ndarray,
    u_gumbel: np.ndarray,
    *,
    temperature_p: float = 1.0,
    temperature_q: float = 1.0,
    sampler_x: float = 0.5,
    alignment: str = "reference",
    return_margins: bool = False,
):
    """verify.py:68-120 with explicit uniforms.

    Returns (accept_until, recovery, accepted_mask) and, with
    ``return_margins``, per-row float64 margins ``(accept_margin, gumbel_gap)``:
    the smallest |u - ratio| over the accept tests taken and the gap between the
    best and second-best Gumbel scores.  Tests treat rows whose margin is below
    the fp32 rounding noise of exp/log as near-ties rather than mismatches.
    """
    b, kp1, v = logits_p.shape
    k = kp1 - 1
    off = 1 if alignment == "reference" else 0
    tp = np.float32(temperature_p)
    tq = np.float32(temperature_q)
    x = np.float32(sampler_x)
    acc_out = np.zeros(b, np.int32)
    rec_out = np.zeros(b, np.int32)
    acc_margin = np.full(b, np.inf)
    gap = np.zeros(b)
    for i in range(b):
        lp = logits_p[i].astype(np.float32)
        lq = logits_q[i].astype(np.float32)
        acc = 0
        for j in range(k):
            p = softmax(lp[j + off] / tp)
            q = softmax(lq[j] / tq)
            tok = int(speculations[i, j + 1])
            ratio = np.minimum(np.float32(1.0), p[tok] / np.maximum(q[tok], np.float32(1e-12)))
            u = np.float32(u_accept[i, j])
            acc_margin[i] = min(acc_margin[i], abs(float(u) - float(ratio)))
            if u < ratio:
                acc += 1
            else:
                break
        if acc == k:
            pf = softmax(lp[k] / tp)
            logit = np.log(pf + np.float32(1e-12))
        else:
            pr = softmax(lp[acc + off] / tp)
            qr = softmax(lq[acc] / tq)
            r = np.maximum(pr - x * qr, np.float32(0.0))
            r = r / np.maximum(r.sum(dtype=np.float32), np.float32(1e-12))
            logit = np.log(r + np.float32(1e-12))
        g = -np.log(-np.log(u_gumbel[i].astype(np.float32)))
        score = (logit + g).astype(np.float32)
        rec = int(np.argmax(score))
        s64 = np.sort(score.astype(np.float64))
        gap[i] = s64[-1] - s64[-2] if v > 1 else np.inf
        acc_out[i] = acc
        rec_out[i] = rec
    mask = np.zeros((b, kp1), dtype=bool)
    mask[:, 1:] = np.arange(k)[None, :] < acc_out[:, None]
    if return_margins:
        return acc_out, rec_out, mask, (acc_margin, gap)
    return acc_out, rec_out, mask
