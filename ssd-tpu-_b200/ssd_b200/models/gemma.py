"""Gemma decoder on the verify-path kernels (replaces the HF Flax Gemma that
jax_ssd/models/gemma_adapter.py:37,61-64,81-102 calls).

Weights live on the GPU in the layout the kernels stream:

* ``w_qkv[l]``      [(Hq + 2*Hkv) * D, d]   rows of Wq, then Wk, then Wv; with
                                            ``qk_pairs`` (opt-in, bf16) each q/k head's rows
                                            are rotation pairs (2i: dim i, 2i+1: dim i + D/2)
* ``w_o[l]``        [d, Hq * D]
* ``w_gate_up[l]``  [2F, d]                 row 2i = gate_i, row 2i+1 = up_i
* ``w_down[l]``     [d, F]
* ``embed``         [V, d]                  also the tied LM head

The input and MLP RMSNorm weights g are folded into the projections that read
the normalised rows: ``w_qkv = W_qkv * (1 + g_attn)`` and ``w_gate_up = W_gu *
(1 + g_mlp)`` column-wise (fp32 product, rounded once to the storage dtype); the
projection kernels scale each token row by its rsqrt(mean(x^2) + eps).  The
norm vectors are kept for reference; the forward does not read them.

Random init (the reference loads checkpoints; the benchmark configs use random
weights from a seed) runs on the device with the counter-based
``ssd_normal_fill``: projections ~ N(0, (1.2/sqrt(fan_in))^2), embedding ~
N(0, 0.005^2), norm weights ~ N(0, 0.1^2).  The small embedding keeps the tied
LM head from echoing the input token, so greedy streams are not degenerate.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from .._lib import GemmaBatchC, GemmaWeightsC, check, dtype_code, lib, ptr, stream_ptr


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

    @property
    def qkv_rows(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim

    def num_params(self) -> int:
        d, f = self.d_model, self.ffn
        per = self.qkv_rows * d + d * self.num_heads * self.head_dim + 3 * d * f + 2 * d
        return self.num_layers * per + self.vocab * d + d

    def layer_weight_bytes(self, elem: int = 2) -> int:
        d, f = self.d_model, self.ffn
        return elem * (self.qkv_rows * d + d * self.num_heads * self.head_dim + 3 * d * f)

    def kv_bytes_per_token(self, elem: int = 2) -> int:
        return elem * 2 * self.num_layers * self.num_kv_heads * self.head_dim


# The model shapes the engine and the benchmark use: the small toy pair (2-layer target, 1-layer draft,
# d_model 256, vocab 1024), the Gemma-7B / Gemma-2B pair, and small bf16 pairs for tensor-parallel checks.
PRESETS = {
    "toy-target": GemmaShape(2, 256, 4, 1, 64, 1024, 1024),
    "toy-draft": GemmaShape(1, 256, 4, 1, 64, 1024, 1024),
    "gemma-7b": GemmaShape(28, 3072, 16, 16, 256, 24576, 256000),
    "gemma-2b": GemmaShape(18, 2048, 8, 1, 256, 16384, 256000),
    # small bf16 pair whose every projection suits the tcgen05 path at 1..8 ranks
    # (tensor-parallel tests): 8 heads of 64, FFN 1024, vocab 2048
    "tp-target": GemmaShape(2, 256, 8, 8, 64, 1024, 2048),
    "tp-draft": GemmaShape(1, 256, 8, 1, 64, 1024, 2048),
}

EMBED_STD = 0.005
NORM_STD = 0.1


def init_std(fan_in: int, gain: float = 1.2) -> float:
    return gain / math.sqrt(fan_in)


def rope_tables(max_pos: int, head_dim: int, theta: float = 10000.0):
    """cos/sin [max_pos, D/2] fp32, computed in float64 on the host and rounded once."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :half]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _mix(seed: int, i: int) -> int:
    z = (seed * 0x9E3779B97F4A7C15 + i * 0xBF58476D1CE4E5B9 + 0x94D049BB133111EB) & (2**64 - 1)
    z ^= z >> 31
    return z


class GemmaWeights:
    """Device-resident Gemma weights in the kernel layout."""

    def __init__(self, shape: GemmaShape, dtype=torch.bfloat16, device="cuda", max_pos: int = 8192):
        self.shape = shape
        self.dtype = dtype
        self.device = torch.device(device)
        s = shape
        z = lambda *sh: torch.empty(sh, dtype=dtype, device=self.device)  # noqa: E731
        self.embed = z(s.vocab, s.d_model)
        self.final_norm = z(s.d_model)
        self.attn_norm = [z(s.d_model) for _ in range(s.num_layers)]
        self.w_qkv = [z(s.qkv_rows, s.d_model) for _ in range(s.num_layers)]
        self.w_o = [z(s.d_model, s.num_heads * s.head_dim) for _ in range(s.num_layers)]
        self.mlp_norm = [z(s.d_model) for _ in range(s.num_layers)]
        self.w_gate_up = [z(2 * s.ffn, s.d_model) for _ in range(s.num_layers)]
        self.w_down = [z(s.d_model, s.ffn) for _ in range(s.num_layers)]
        cos, sin = rope_tables(max_pos, s.head_dim, s.rope_theta)
        self.rope_cos = torch.from_numpy(cos).to(self.device)
        self.rope_sin = torch.from_numpy(sin).to(self.device)
        self.max_pos = max_pos
        self.tp_rank, self.tp_world = 0, 1  # set by runtime.tensor_parallel.shard_weights
        # True: the q and k rows of every head are stored as rotation pairs (see pair_qk_rows)
        self.qk_pairs = False
        self._cstruct = None

    # ------------------------------------------------------------ init
    def _fill(self, t: torch.Tensor, std: float, seed: int) -> None:
        check(lib().ssd_normal_fill(stream_ptr(), ptr(t), dtype_code(t.dtype), t.numel(), float(std),
                                    seed & (2**64 - 1)), "ssd_normal_fill")

    @classmethod
    def random(cls, shape: GemmaShape, seed: int, dtype=torch.bfloat16, device="cuda",
               max_pos: int = 8192) -> "GemmaWeights":
        w = cls(shape, dtype, device, max_pos)
        s = shape
        i = 0

        def nxt():
            nonlocal i
            i += 1
            return _mix(seed, i)

        w._fill(w.embed, EMBED_STD, nxt())
        w._fill(w.final_norm, NORM_STD, nxt())
        for l in range(s.num_layers):
            w._fill(w.attn_norm[l], NORM_STD, nxt())
            w._fill(w.w_qkv[l], init_std(s.d_model), nxt())
            w._fill(w.w_o[l], init_std(s.num_heads * s.head_dim), nxt())
            w._fill(w.mlp_norm[l], NORM_STD, nxt())
            w._fill(w.w_gate_up[l], init_std(s.d_model), nxt())
            w._fill(w.w_down[l], init_std(s.ffn), nxt())
        w._fold_norms()
        return w

    def pair_qk_rows(self) -> "GemmaWeights":
        """Store the q and k rows of every head as rotation pairs: row 2i = dimension i,
        row 2i+1 = dimension i + D/2 (v rows unchanged).  The bf16 forward then applies
        RoPE and writes the K/V rows in the QKV projection's epilogue, where both halves
        of a pair sit in adjacent lanes (``ssd_gemma_weights.qk_pairs``), instead of
        running the separate RoPE + K/V write kernel.  Opt-in: in the 7B/2B decode loop
        the separate kernel measured faster (89.6 vs 86.4 tok/s on one B200)."""
        if self.qk_pairs:
            return self
        if self.dtype != torch.bfloat16:
            raise ValueError("q/k rotation pairs need bf16 weights (the tcgen05 projection)")
        s = self.shape
        D, d = s.head_dim, s.d_model
        for l in range(s.num_layers):
            qk = self.w_qkv[l][:(s.num_heads + s.num_kv_heads) * D]
            heads = s.num_heads + s.num_kv_heads
            qk.copy_(qk.view(heads, 2, D // 2, d).transpose(1, 2).reshape(heads * D, d).clone())
        self.qk_pairs = True
        self._cstruct = None
        return self

    def _fold_norms(self) -> None:
        """w_qkv *= (1 + attn_norm), w_gate_up *= (1 + mlp_norm) column-wise (fp32, rounded once)."""
        for l in range(self.shape.num_layers):
            for mat, g in ((self.w_qkv[l], self.attn_norm[l]), (self.w_gate_up[l], self.mlp_norm[l])):
                mat.copy_((mat.float() * (1.0 + g.float())[None, :]).to(self.dtype))

    @classmethod
    def from_canonical(cls, shape: GemmaShape, host: dict, dtype=torch.bfloat16, device="cuda",
                       max_pos: int = 8192, qk_pairs: bool = False) -> "GemmaWeights":
        """Pack canonical per-matrix weights (wq/wk/wv/wo/wg/wu/wd, numpy or torch).

        ``qk_pairs`` stores the q/k rows as rotation pairs (``pair_qk_rows``)."""
        w = cls(shape, dtype, device, max_pos)
        t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.float32)).to(device=w.device, dtype=dtype)  # noqa: E731
        w.embed.copy_(t(host["embed"]))
        w.final_norm.copy_(t(host["final_norm"]))
        for l, lw in enumerate(host["layers"]):
            w.attn_norm[l].copy_(t(lw["attn_norm"]))
            w.mlp_norm[l].copy_(t(lw["mlp_norm"]))
            w.w_qkv[l].copy_(torch.cat([t(lw["wq"]), t(lw["wk"]), t(lw["wv"])], 0))
            w.w_o[l].copy_(t(lw["wo"]))
            gu = torch.stack([t(lw["wg"]), t(lw["wu"])], 1).reshape(2 * shape.ffn, shape.d_model)
            w.w_gate_up[l].copy_(gu)
            w.w_down[l].copy_(t(lw["wd"]))
        if not host.get("folded", False):
            w._fold_norms()
        if qk_pairs:
            w.pair_qk_rows()
        return w

    def to_canonical(self, layers: int | None = None) -> dict:
        """Unpack to per-matrix float32 numpy arrays (for the CPU oracle).

        The q/k/v and gate/up matrices are returned as stored, i.e. with the
        RMSNorm weights folded in (``"folded": True``).
        """
        s = self.shape
        f = lambda x: x.float().cpu().numpy()  # noqa: E731
        out = {"embed": f(self.embed), "final_norm": f(self.final_norm), "layers": [], "folded": True}
        for l in range(s.num_layers if layers is None else layers):
            out["layers"].append(self.canonical_layer(l))
        return out

    def canonical_layer(self, l: int) -> dict:
        """Layer ``l`` of ``to_canonical`` alone (float32 numpy)."""
        s = self.shape
        f = lambda x: x.float().cpu().numpy()  # noqa: E731
        hq, hkv = s.num_heads * s.head_dim, s.num_kv_heads * s.head_dim
        qkv = f(self.w_qkv[l])
        if self.qk_pairs:  # back to canonical row order
            heads, D = s.num_heads + s.num_kv_heads, s.head_dim
            qkv[:heads * D] = (qkv[:heads * D].reshape(heads, D // 2, 2, s.d_model)
                               .transpose(0, 2, 1, 3).reshape(heads * D, s.d_model))
        gu = f(self.w_gate_up[l]).reshape(s.ffn, 2, s.d_model)
        return {"attn_norm": f(self.attn_norm[l]), "mlp_norm": f(self.mlp_norm[l]),
                "wq": np.ascontiguousarray(qkv[:hq]), "wk": np.ascontiguousarray(qkv[hq:hq + hkv]),
                "wv": np.ascontiguousarray(qkv[hq + hkv:]), "wo": f(self.w_o[l]),
                "wg": np.ascontiguousarray(gu[:, 0]), "wu": np.ascontiguousarray(gu[:, 1]), "wd": f(self.w_down[l])}

    # ------------------------------------------------------------ C view
    def cstruct(self) -> GemmaWeightsC:
        if self._cstruct is None:
            s = self.shape
            arr = lambda ts: (C.c_void_p * len(ts))(*[ptr(t) for t in ts])  # noqa: E731
            self._arrays = [arr(self.w_qkv), arr(self.w_o), arr(self.w_gate_up), arr(self.w_down)]
            cs = GemmaWeightsC()
            cs.num_layers, cs.d_model, cs.num_heads, cs.num_kv_heads = s.num_layers, s.d_model, s.num_heads, s.num_kv_heads
            cs.head_dim, cs.ffn, cs.vocab, cs.eps = s.head_dim, s.ffn, s.vocab, s.eps
            cs.dtype = dtype_code(self.dtype)
            cs.embed, cs.final_norm = ptr(self.embed), ptr(self.final_norm)
            P = C.POINTER(C.c_void_p)
            cs.w_qkv, cs.w_o, cs.w_gate_up, cs.w_down = [C.cast(a, P) for a in self._arrays]
            cs.rope_cos, cs.rope_sin, cs.rope_max_pos = ptr(self.rope_cos), ptr(self.rope_sin), self.max_pos
            cs.tp_rank, cs.tp_world = self.tp_rank, self.tp_world
            cs.qk_pairs = int(self.qk_pairs)
            self._cstruct = cs
        return self._cstruct

    def weight_bytes(self) -> int:
        es = 2 if self.dtype == torch.bfloat16 else 4
        return self.shape.num_params() * es


class GemmaRunner:
    """One ``ssd_gemma_forward`` per call; scratch sized for (max_batch, max_tokens).

    With ``comm`` (a ``runtime.tensor_parallel.TPComm``) the weights are one
    rank's shard and the logits buffers passed to ``forward`` must come from
    ``comm.alloc`` (the LM head all-gathers into them).
    """

    def __init__(self, weights: GemmaWeights, max_batch: int, max_tokens: int, max_seq_len: int, comm=None):
        self.w = weights
        self.max_batch = max_batch
        self.max_tokens = max_tokens
        self.max_seq_len = max_seq_len
        self.comm = comm
        if weights.tp_world > 1 and comm is None:
            raise ValueError("sharded weights need the tensor-parallel comm")
        self._comm_ptr = C.pointer(comm.cstruct) if comm is not None else None
        self._scratch = {}

    def scratch(self, b: int, t: int) -> torch.Tensor:
        key = (b, t)
        buf = self._scratch.get(key)
        if buf is None:
            n = lib().ssd_gemma_scratch_size(C.byref(self.w.cstruct()), b, t, self.max_seq_len)
            buf = torch.zeros(n, dtype=torch.uint8, device=self.w.device)
            self._scratch[key] = buf
        return buf

    def forward(self, tokens: torch.Tensor, seq_lens_before: torch.Tensor, pages: torch.Tensor,
                block_tables: torch.Tensor, logits: torch.Tensor | None, q_lens: torch.Tensor | None = None,
                last_only: bool = False, stream=None, prof: "ProjectionTimer | None" = None) -> torch.Tensor:
        b, t = tokens.shape
        sc = self.scratch(b, t)
        bt = GemmaBatchC()
        bt.B, bt.T = b, t
        bt.tokens, bt.seq_lens_before, bt.q_lens = ptr(tokens), ptr(seq_lens_before), ptr(q_lens)
        bt.kv_pages = ptr(pages)
        bt.num_blocks, bt.block_size = pages.shape[2], pages.shape[3]
        bt.block_tables, bt.max_blocks = ptr(block_tables), block_tables.shape[1]
        bt.max_seq_len = self.max_seq_len
        bt.logits, bt.logits_last_only = ptr(logits), int(bool(last_only))
        bt.scratch, bt.scratch_bytes = ptr(sc), sc.numel()
        bt.comm = self._comm_ptr
        if prof is not None:
            prof.attach(bt)
        check(lib().ssd_gemma_forward(stream_ptr(stream), C.byref(self.w.cstruct()), C.byref(bt)),
              "ssd_gemma_forward")
        if prof is not None:
            prof.collect()
        return logits

    @staticmethod
    def launches_per_forward(shape: GemmaShape, with_logits: bool, last_only: bool) -> int:
        """Kernel launches issued by one ssd_gemma_forward (positions, embed, 6 per layer, head)."""
        n = 2 + 8 * shape.num_layers
        if with_logits:
            n += 2 + (1 if last_only else 0)
        return n


class ProjectionTimer:
    """CUDA events around every projection launch of a forward (ssd_gemma_batch.prof_*).

    ``attach`` binds the event array into the batch struct; the C++ forward
    records event 2i / 2i+1 around its i-th projection (also inside a captured
    CUDA graph, where the records become graph nodes).  ``read`` — called after
    the step has synchronised — adds the elapsed time of the bound pairs.
    """

    KINDS = ("qkv", "o", "gate_up", "down", "lm_head")

    def __init__(self, capacity: int = 512):
        self.capacity = capacity
        self.events = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(2 * capacity)]
        st = torch.cuda.current_stream()
        for e in self.events:
            e.record(st)  # materialise the handles
        torch.cuda.synchronize()
        self._arr = (C.c_void_p * (2 * capacity))(*[e.cuda_event for e in self.events])
        self._count = C.c_int(0)
        self._kind = (C.c_int * capacity)()
        self.bound = []
        self.total_ms = {k: 0.0 for k in self.KINDS}
        self.launches = {k: 0 for k in self.KINDS}

    def attach(self, bt) -> None:
        bt.prof_events = C.cast(self._arr, C.POINTER(C.c_void_p))
        bt.prof_capacity = self.capacity
        bt.prof_count = C.pointer(self._count)
        bt.prof_kind = C.cast(self._kind, C.POINTER(C.c_int))

    def collect(self) -> None:
        self.bound = [(self.KINDS[self._kind[i]], self.events[2 * i], self.events[2 * i + 1])
                      for i in range(self._count.value)]

    def read(self) -> None:
        for kind, a, b in self.bound:
            self.total_ms[kind] += a.elapsed_time(b)
            self.launches[kind] += 1

    def reset(self) -> None:
        self.total_ms = {k: 0.0 for k in self.KINDS}
        self.launches = {k: 0 for k in self.KINDS}
