"""Oracle: Gemma decoder forward over a paged KV cache (test infrastructure only).

The reference delegates the Gemma arithmetic to the third-party HF
``FlaxAutoModelForCausalLM`` (``jax_ssd/models/gemma_adapter.py:37,61-64,89-94``;
``transformers>=4.48.0``, unpinned, not vendored; transformers 5.x has no Flax).
This module restates the published Gemma-1 architecture:

* embedding ``x = E[tok] * sqrt(d)``;
* ``RMSNorm(x) = x * rsqrt(mean(x^2) + 1e-6) * (1 + w)``;
* q/k/v projections, rotary embedding (theta 10000, rotate-half pairing of
  dim ``i`` with ``i + D/2``), attention with scale ``1/sqrt(D)`` over the
  paged cache (``paged_kv.paged_verify_attention``), output projection;
* GeGLU MLP ``down(gelu_tanh(gate(x)) * up(x))``;
* final RMSNorm and the tied LM head ``logits = h E^T``.

Weights may come "folded" (``weights["folded"]``): the q/k/v and gate/up
matrices then already carry the RMSNorm weights, ``W' = W * (1 + g)``
column-wise, and those projections compute ``round(inv(x) * (x @ W'^T))`` with
``inv(x) = 1/sqrt(mean(x^2) + eps)`` -- the formulation the CUDA path uses.
Unfolded weights use the textbook ``round(round(norm(x)) @ W^T)``; in fp32 the
two agree to rounding.

``precision="fp32"`` computes everything in float32 (the toy pair, and the
cross-check against the installed torch ``GemmaForCausalLM``).
``precision="bf16"`` rounds to bfloat16 at exactly the points where the CUDA
path stores bf16: after the embedding scale, each RMSNorm, each projection,
RoPE, attention, GeGLU and each residual add.  Logits stay fp32.
Parity unpinned: no reference run of the Gemma forward is possible here.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import paged_kv


@dataclass(frozen=True)
class GemmaShape:
    num_layers: int
    d_model: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 10000.0


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def rope_table(max_pos: int, head_dim: int, theta: float = 10000.0):
    """cos/sin [max_pos, head_dim/2] in float32 (computed in float64, rounded once).

    The CUDA path uploads this same table, so both sides rotate with identical
    coefficients.
    """
    half = head_dim // 2
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :half]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    c = np.float32(np.sqrt(2.0 / np.pi))
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


def init_std(fan_in: int, gain: float = 1.2) -> float:
    """Projection init scale: ``gain / sqrt(fan_in)``."""
    return gain / float(np.sqrt(fan_in))


EMBED_STD = 0.005
NORM_STD = 0.1


def init_weights(shape: GemmaShape, seed: int) -> dict:
    """Seeded random init (numpy default_rng), float32; small models only.

    Projections ~ N(0, (1.2/sqrt(fan_in))^2), embedding ~ N(0, 0.005^2), norm
    weights ~ N(0, 0.1^2).  The small embedding keeps the tied LM head from
    simply echoing the input token, so greedy streams are not degenerate.
    """
    rng = np.random.default_rng(seed)
    d, hq, hkv, hd, f = shape.d_model, shape.num_heads, shape.num_kv_heads, shape.head_dim, shape.ffn

    def n(*s, sd):
        return (rng.standard_normal(s, dtype=np.float32) * np.float32(sd)).astype(np.float32)

    w = {"embed": n(shape.vocab, d, sd=EMBED_STD), "final_norm": n(d, sd=NORM_STD), "layers": []}
    for _ in range(shape.num_layers):
        w["layers"].append({
            "attn_norm": n(d, sd=NORM_STD), "wq": n(hq * hd, d, sd=init_std(d)),
            "wk": n(hkv * hd, d, sd=init_std(d)), "wv": n(hkv * hd, d, sd=init_std(d)),
            "wo": n(d, hq * hd, sd=init_std(hq * hd)), "mlp_norm": n(d, sd=NORM_STD),
            "wg": n(f, d, sd=init_std(d)), "wu": n(f, d, sd=init_std(d)), "wd": n(d, f, sd=init_std(f)),
        })
    return w


class OracleGemma:
    def __init__(self, shape: GemmaShape, weights: dict, precision: str = "fp32", max_pos: int = 8192):
        self.s = shape
        self.bf = precision == "bf16"
        r = bf16_round if self.bf else (lambda a: a.astype(np.float32))
        self.r = r
        layers = weights["layers"]
        # a callable fetches layer i on demand (full-depth checks of large models keep one layer
        # in host memory at a time); its arrays must already be representable in the precision
        self._layer_fn = layers if callable(layers) else None
        self.w = {
            "embed": r(weights["embed"]),
            "final_norm": r(weights["final_norm"]),
            "layers": None if self._layer_fn else [{k: r(v) for k, v in lw.items()} for lw in layers],
        }
        self.cos, self.sin = rope_table(max_pos, shape.head_dim, shape.rope_theta)
        self.folded = bool(weights.get("folded", False))

    # ---- pieces (each rounds where the CUDA path stores bf16)
    def embed(self, tokens):
        scale = np.float32(np.sqrt(self.s.d_model))
        if self.bf:
            scale = bf16_round(np.array([scale], np.float32))[0]
        return self.r(self.w["embed"][tokens] * scale)

    def rmsnorm(self, x, w):
        xf = x.astype(np.float32)
        ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
        y = xf * (np.float32(1.0) / np.sqrt(ms + np.float32(self.s.eps))) * (np.float32(1.0) + w)
        return self.r(y)

    def linear(self, x, w):
        return self.r(x.astype(np.float32) @ w.T)

    def row_parallel(self, x, w, allreduce=None):
        """round(x @ w^T), the fp32 product summed over the ranks first when sharded."""
        y = x.astype(np.float32) @ w.T
        if allreduce is not None:
            y = allreduce(y.astype(np.float32))
        return self.r(y)

    def inv_rms(self, x):
        xf = x.astype(np.float32)
        ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
        return (np.float32(1.0) / np.sqrt(ms + np.float32(self.s.eps))).astype(np.float32)

    def linear_rownorm(self, x, w):
        """round(inv(x) * (x @ w^T)) for folded weights."""
        return self.r((x.astype(np.float32) @ w.T) * self.inv_rms(x))

    def rope(self, x, pos):
        """x[..., H, D] at positions pos[...] (same leading shape)."""
        half = self.s.head_dim // 2
        c = self.cos[pos][..., None, :]
        s = self.sin[pos][..., None, :]
        x1, x2 = x[..., :half].astype(np.float32), x[..., half:].astype(np.float32)
        return self.r(np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1))

    def forward(self, tokens, pages, block_tables, seq_lens_before, q_lens=None, stop_layer=None, timings=None,
                with_head=True, allreduce=None, allgather=None, vocab_block=None):
        """tokens[B,T] -> logits[B,T,V] fp32; writes K/V of the new tokens into ``pages``.

        Sequence b's new token t (t < q_lens[b]) sits at position
        ``seq_lens_before[b] + t``.  ``pages`` is [2,L,NB,BS,Hkv,D] float32 holding
        bf16-representable values in bf16 mode.

        Tensor-parallel restatement (the sharded CUDA forward): with the
        weights of one rank's shard, ``allreduce(partial_fp32)`` sums the O and
        down partial products over the ranks before they are rounded and added
        to the residual, and the LM head multiplies by the rows
        ``vocab_block = (v0, nv)`` of the embedding and ``allgather``s the
        column blocks.
        """
        s = self.s
        bsz, t = tokens.shape
        ql = np.full(bsz, t, np.int64) if q_lens is None else np.asarray(q_lens, np.int64)
        pos = np.asarray(seq_lens_before, np.int64)[:, None] + np.arange(t)[None, :]
        valid = np.arange(t)[None, :] < ql[:, None]
        wpos = np.where(valid, pos, -1)
        seq_after = np.asarray(seq_lens_before, np.int64) + ql
        import time as _time

        t_start = _time.perf_counter()
        x = self.embed(tokens)  # [B,T,d]
        nl = s.num_layers if stop_layer is None else stop_layer
        for li in range(nl):
            lw = self._layer_fn(li) if self._layer_fn else self.w["layers"][li]
            if self.folded:
                proj, h = self.linear_rownorm, x
            else:
                proj, h = self.linear, self.rmsnorm(x, lw["attn_norm"])
            q = proj(h, lw["wq"]).reshape(bsz, t, s.num_heads, s.head_dim)
            k = proj(h, lw["wk"]).reshape(bsz, t, s.num_kv_heads, s.head_dim)
            v = proj(h, lw["wv"]).reshape(bsz, t, s.num_kv_heads, s.head_dim)
            pc = np.where(valid, pos, 0)
            q = self.rope(q, pc)
            k = self.rope(k, pc)
            paged_kv.write_kv(pages, li, block_tables, wpos, k, v)
            a = paged_kv.paged_verify_attention(q, pages, li, block_tables, seq_after, ql)
            a = self.r(a.astype(np.float32)).reshape(bsz, t, s.num_heads * s.head_dim)
            x = self.r(x + self.row_parallel(a, lw["wo"], allreduce))
            if self.folded:
                g = self.linear_rownorm(x, lw["wg"])
                u = self.linear_rownorm(x, lw["wu"])
            else:
                h = self.rmsnorm(x, lw["mlp_norm"])
                g = self.linear(h, lw["wg"])
                u = self.linear(h, lw["wu"])
            m = self.r(self.r(gelu_tanh(g)) * u)
            x = self.r(x + self.row_parallel(m, lw["wd"], allreduce))
        t_layers = _time.perf_counter()
        if not with_head:
            return None
        h = self.rmsnorm(x, self.w["final_norm"])
        head = self.w["embed"] if vocab_block is None else self.w["embed"][vocab_block[0]:vocab_block[0] + vocab_block[1]]
        out = (h.astype(np.float32) @ head.T).astype(np.float32)
        if allgather is not None:
            out = allgather(out)
        if timings is not None:  # wall-clock split used by the CPU baseline
            timings["layers_s"] = t_layers - t_start
            timings["head_s"] = _time.perf_counter() - t_layers
        return out


def fold_norms(weights: dict) -> dict:
    """Fold the RMSNorm weights into q/k/v and gate/up (fp32): W' = W * (1 + g) column-wise."""
    out = {"embed": weights["embed"], "final_norm": weights["final_norm"], "layers": [], "folded": True}
    for lw in weights["layers"]:
        a = (np.float32(1.0) + lw["attn_norm"].astype(np.float32))[None, :]
        m = (np.float32(1.0) + lw["mlp_norm"].astype(np.float32))[None, :]
        out["layers"].append({**lw, "wq": lw["wq"] * a, "wk": lw["wk"] * a, "wv": lw["wv"] * a,
                              "wg": lw["wg"] * m, "wu": lw["wu"] * m})
    return out


def new_pages(shape: GemmaShape, num_blocks: int, block_size: int) -> np.ndarray:
    return np.zeros((2, shape.num_layers, num_blocks, block_size, shape.num_kv_heads, shape.head_dim), np.float32)


def greedy_ar(model: OracleGemma, prompt, max_new: int, num_blocks: int = 64, block_size: int = 16):
    """Target-only greedy decode (the AR loop of ``jax_ssd/runtime/engine.py:162-211``)."""
    pages = new_pages(model.s, num_blocks, block_size)
    table = np.arange(num_blocks, dtype=np.int32)[None, :]
    toks = np.asarray(prompt, np.int64)[None, :]
    logits = model.forward(toks, pages, table, [0])
    out = [int(np.argmax(logits[0, -1]))]
    n = len(prompt)
    while len(out) < max_new:
        logits = model.forward(np.array([[out[-1]]]), pages, table, [n])
        n += 1
        out.append(int(np.argmax(logits[0, -1])))
    return out
