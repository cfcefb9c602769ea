"""Speculative decoding of B sequences at once (batched serving).

The reference decodes one prompt at a time (jax_ssd/runtime/engine.py:110-125);
this decoder runs B sequences through every kernel together, which is what
makes the verify forward's projections wider than a few rows and what the
batched serving workload (B = 32, k = 6, sampling) measures.

Per step, for all B sequences (all device work stream-ordered, one host sync):

1. rollback of the previous step on both caches, one call each
   (``ssd_page_rollback`` over B rows, per-sequence lengths);
2. draft: one forward over each sequence's 1-2 not yet drafted tokens (ragged
   ``q_lens``), then k-1 one-token forwards; each draft token is the argmax
   (temperature 0) or a Gumbel-max draw from softmax(logits / T)
   (``ssd_sample_rows``), restricted to the top-p nucleus when ``top_p < 1``
   (``ssd_top_p_mask`` on the draft rows in place); in sampling mode the
   (masked) draft rows are kept for the acceptance test;
3. verify: one target forward over B x (k+1) tokens (its rows top-p masked
   likewise in sampling mode);
4. acceptance: ``ssd_verify_greedy`` or ``ssd_verify_sample`` (rejection
   sampling with bonus / residual draw, the textbook row alignment) over the B
   rows;
5. one device->host copy of (accepted, recovery, verify tokens) for all rows.

Greedy mode is batch invariant: each sequence's stream equals its one-sequence
greedy decode exactly.
"""

from __future__ import annotations

import numpy as np
import torch

from .._lib import check, lib, ptr, stream_ptr
from ..algorithm.verify import argmax_rows, sample_rows, top_p_mask_, verify_sample
from ..kernels.kv_cache import KVCacheState
from ..kernels.ops import max_tokens_per_forward
from ..models.gemma import GemmaRunner, GemmaWeights
from ..workspace import workspace
from .page_manager import PageManager


class _BatchModel:
    def __init__(self, weights: GemmaWeights, batch: int, max_seq_len: int, block_size: int, tokens: int,
                 comm=None, num_blocks: int | None = None):
        s = weights.shape
        self.w = weights
        self.max_blocks = (max_seq_len + block_size - 1) // block_size + 1
        self.num_blocks = num_blocks or batch * self.max_blocks + 2
        self.cache = KVCacheState.allocate(s.num_layers, self.num_blocks, block_size, s.num_kv_heads, s.head_dim,
                                           dtype=weights.dtype, device=weights.device)
        self.pm = PageManager(block_size, self.num_blocks, max_seqs=batch, max_blocks_per_seq=self.max_blocks,
                              device=weights.device)
        self.runner = GemmaRunner(weights, batch, tokens, max_seq_len, comm=comm)
        self.chunk = min(64, max_tokens_per_forward(weights.dtype))
        self.n = np.zeros(batch, np.int64)  # tokens cached per sequence


class BatchedSpeculativeDecoder:
    def __init__(self, target: GemmaWeights, draft: GemmaWeights, batch: int, k: int = 4, max_seq_len: int = 1024,
                 block_size: int = 16, temperature: float = 0.0, sampler_x: float = 0.5, seed: int = 0, comm=None,
                 num_blocks: int | None = None, top_p: float = 1.0):
        B = self.B = int(batch)
        self.k = k
        self.temperature = float(temperature)
        self.top_p = float(top_p)
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        self.sampler_x = float(sampler_x)
        self.seed = int(seed)
        self.dev = target.device
        V = self.V = target.shape.vocab
        if draft.shape.vocab != V:
            raise ValueError("target and draft must share the vocabulary")
        if B * (k + 1) > max_tokens_per_forward(target.dtype):
            raise ValueError(f"B*(k+1) = {B * (k + 1)} exceeds one forward ({max_tokens_per_forward(target.dtype)})")
        self.t = _BatchModel(target, B, max_seq_len, block_size, max(k + 1, 64), comm, num_blocks)
        self.d = _BatchModel(draft, B, max_seq_len, block_size, 64, comm, num_blocks)
        dev = self.dev
        buf = comm.alloc if comm is not None else (lambda shape, dtype: torch.empty(shape, dtype=dtype, device=dev))
        self.vt = torch.zeros((B, k + 1), dtype=torch.int32, device=dev)      # [recovery, drafts...]
        self.dtok = torch.zeros((k, B), dtype=torch.int32, device=dev)        # draft token i of every sequence
        self.feed = torch.zeros((B, 2), dtype=torch.int32, device=dev)
        self.logits_t = buf((B, k + 1, V), torch.float32)
        self.logits_d = buf((B, V), torch.float32)
        self.sampling = self.temperature > 0
        if self.sampling:
            self.logits_q = torch.empty((B, k, V), dtype=torch.float32, device=dev)
            self.u_accept = torch.empty((B, k), dtype=torch.float32, device=dev)
            self.u_gumbel = torch.empty((B, V), dtype=torch.float32, device=dev)
        self.acc = torch.zeros(B, dtype=torch.int32, device=dev)
        self.rec = torch.zeros(B, dtype=torch.int32, device=dev)
        self.mask = torch.empty((B, k + 1), dtype=torch.uint8, device=dev)
        self.ws_greedy = workspace(dev, "bsd_greedy", lib().ssd_verify_greedy_workspace_size(B, k, V))
        # host -> device scalars of one step, one pinned copy: 12 + k - 1 rows of B int32
        self.nrow = 12 + k
        self.h_scal = torch.zeros((self.nrow, B), dtype=torch.int32).pin_memory()
        self.d_scal = torch.zeros((self.nrow, B), dtype=torch.int32, device=dev)
        self.h_out = torch.zeros((2 + k + 1, B), dtype=torch.int32).pin_memory()
        self.d_out = torch.zeros((2 + k + 1, B), dtype=torch.int32, device=dev)
        self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self.seqs: list[list[int]] = [[] for _ in range(B)]
        self.out: list[list[int]] = [[] for _ in range(B)]
        self._roll = np.zeros((4, B), np.int64)
        self._rec = np.zeros(B, np.int64)
        self._draws = 0
        self.last_accept = np.zeros(B, np.int64)
        self.last_verify_ms = 0.0

    # ------------------------------------------------------------------ set-up
    def _i32(self, v) -> torch.Tensor:
        return torch.as_tensor(np.asarray(v, np.int32)).to(self.dev)

    def _prefill(self, m: _BatchModel, b: int, prompt: list[int], want_logits: bool) -> None:
        n = len(prompt)
        p = torch.tensor([prompt], dtype=torch.int32, device=self.dev)
        m.pm.allocate_rows(b, 1, self._i32([0]), self._i32([n]), None)
        for c0 in range(0, n, m.chunk):
            c1 = min(n, c0 + m.chunk)
            lg = self.logits_d[b:b + 1] if (c1 == n and want_logits) else None
            m.runner.forward(p[:, c0:c1].contiguous(), self._i32([c0]), m.cache.pages, m.pm.tables[b:b + 1], lg,
                             last_only=True)
        m.n[b] = n

    def admit(self, b: int, prompt: list[int]) -> int:
        """Seat ``prompt`` in row ``b`` (continuous batching): release the row's pages in both
        caches, prefill it on both models, and return its first token (target argmax).  The
        other rows keep their state; the next ``step`` decodes all rows together."""
        prompt = [int(t) for t in prompt]
        if not prompt:
            raise ValueError("empty prompt")
        for m in (self.t, self.d):
            m.pm.free_rows(b, 1)
            m.n[b] = 0
        self._prefill(self.t, b, prompt, True)
        first = torch.empty(1, dtype=torch.int32, device=self.dev)
        argmax_rows(self.logits_d[b:b + 1], first)
        self._prefill(self.d, b, prompt, False)
        f = int(first.item())
        self.seqs[b] = prompt + [f]
        self.out[b] = [f]
        self._roll[:, b] = (self.t.n[b], 0, self.d.n[b], 0)
        self._rec[b] = f
        self.last_accept[b] = 0
        return f

    def park(self, b: int) -> None:
        """Put row ``b`` on a one-token placeholder sequence (a finished row with nothing to
        replace it keeps stepping with the batch; its tokens are not used)."""
        self.admit(b, [0])

    def start(self, prompts: list[list[int]]) -> list[int]:
        """Prefill every sequence on both models; returns each one's first token (target argmax)."""
        if len(prompts) != self.B:
            raise ValueError(f"expected {self.B} prompts")
        return [self.admit(b, pr) for b, pr in enumerate(prompts)]

    def start_synthetic(self, contexts: list[int], rng: np.random.Generator) -> None:
        """Stand-in for a long prefill: allocate each sequence's context pages and fill both caches
        with N(0, 1) K/V (seeded); sequences get random token ids.  Used to measure decode steps
        at long contexts without spending minutes on prefill."""
        V = self.V
        for m in (self.t, self.d):
            m.pm.allocate_rows(0, self.B, self._i32(np.zeros(self.B)), self._i32(contexts), None)
            m.n[:] = np.asarray(contexts, np.int64)
            c = m.cache.pages
            check(lib().ssd_normal_fill(stream_ptr(), ptr(c), 0 if c.dtype == torch.bfloat16 else 1, c.numel(),
                                        1.0, int(rng.integers(1, 2**62))), "ssd_normal_fill")
        for b, n in enumerate(contexts):
            self.seqs[b] = [int(x) for x in rng.integers(0, V, int(n) + 1)]
            self.out[b] = [self.seqs[b][-1]]
        self.d.n[:] = np.asarray(contexts, np.int64)
        self._roll = np.stack([self.t.n, np.zeros(self.B, np.int64), self.d.n, np.zeros(self.B, np.int64)])
        self._rec = np.asarray([s[-1] for s in self.seqs], np.int64)

    # ------------------------------------------------------------------ one step
    # host scalar rows: 0 t_roll_num | 1 t_roll_acc | 2 d_roll_num | 3 d_roll_acc | 4 recovery
    #  5 draft cached | 6 draft reserve | 7 draft feed length | 8-9 feed tokens | 10 target cached
    #  11 k+1 | 12.. draft forward i (i = 1..k-1): tokens cached before it
    def _host_scalars(self) -> np.ndarray:
        k, B = self.k, self.B
        h = self.h_scal.numpy()
        nf = np.zeros(B, np.int64)
        for b in range(B):
            feed = self.seqs[b][int(self.d.n[b]):]
            nf[b] = len(feed)
            h[8, b] = feed[0]
            h[9, b] = feed[1] if len(feed) > 1 else 0
        h[0:4] = self._roll
        h[4] = self._rec
        h[5] = self.d.n
        h[6] = nf + k - 1
        h[7] = nf
        h[10] = self.t.n
        h[11] = k + 1
        for i in range(1, k):
            h[11 + i] = self.d.n + nf + i - 1
        return nf

    def step(self) -> list[list[int]]:
        k, B, t, d = self.k, self.B, self.t, self.d
        nf = self._host_scalars()
        two = int(nf.max()) if B else 1
        ds = self.d_scal
        ds.copy_(self.h_scal, non_blocking=True)
        t.pm.rollback_rows(0, B, ds[0], ds[1])
        d.pm.rollback_rows(0, B, ds[2], ds[3])
        self.vt[:, 0].copy_(ds[4])
        self.feed.copy_(ds[8:10].t())
        # draft
        d.pm.allocate_rows(0, B, ds[5], ds[6], None)
        for i in range(k):
            if i == 0:
                d.runner.forward(self.feed[:, :two].contiguous() if two == 1 else self.feed, ds[5], d.cache.pages,
                                 d.pm.tables, self.logits_d, q_lens=ds[7], last_only=True)
            else:
                d.runner.forward(self.dtok[i - 1].view(B, 1), ds[11 + i], d.cache.pages, d.pm.tables, self.logits_d,
                                 last_only=True)
            if self.sampling:
                if self.top_p < 1.0:
                    top_p_mask_(self.logits_d, self.temperature, self.top_p)
                sample_rows(self.logits_d, self.temperature, self.seed, self._draws * B * self.V, out=self.dtok[i])
                self._draws += 1
                self.logits_q[:, i].copy_(self.logits_d)
            else:
                argmax_rows(self.logits_d, self.dtok[i])
        self.vt[:, 1:].copy_(self.dtok.t())
        # verify
        st = torch.cuda.current_stream()
        self.ev[0].record(st)
        t.pm.allocate_rows(0, B, ds[10], ds[11], None)
        t.runner.forward(self.vt, ds[10], t.cache.pages, t.pm.tables, self.logits_t, last_only=False)
        if self.sampling and self.top_p < 1.0:
            top_p_mask_(self.logits_t.view(B * (k + 1), self.V), self.temperature, self.top_p)
        if self.sampling:
            for u in (self.u_accept, self.u_gumbel):
                check(lib().ssd_uniform_fill(stream_ptr(), ptr(u), u.numel(), self.seed ^ 0x5D5D,
                                             self._draws * B * self.V), "ssd_uniform_fill")
                self._draws += 1
            r = verify_sample(self.logits_t, self.logits_q, self.vt, (self.u_accept, self.u_gumbel),
                              temperature_p=self.temperature, temperature_q=self.temperature,
                              sampler_x=self.sampler_x, alignment="standard")
            self.acc.copy_(r.accept_until)
            self.rec.copy_(r.recovery_tokens)
        else:
            check(lib().ssd_verify_greedy(stream_ptr(), ptr(self.logits_t), ptr(self.vt), ptr(self.acc),
                                          ptr(self.rec), ptr(self.mask), None, ptr(self.ws_greedy),
                                          self.ws_greedy.numel(), B, k, self.V), "ssd_verify_greedy")
        self.ev[1].record(st)
        self.d_out[0].copy_(self.acc)
        self.d_out[1].copy_(self.rec)
        self.d_out[2:].copy_(self.vt.t())
        self.h_out.copy_(self.d_out, non_blocking=True)
        st.synchronize()
        self.last_verify_ms = self.ev[0].elapsed_time(self.ev[1])
        ho = self.h_out.numpy()
        acc = ho[0].astype(np.int64)
        rec = ho[1].astype(np.int64)
        new_all = []
        old_len = np.asarray([len(s) for s in self.seqs], np.int64)
        self._roll = np.stack([t.n.copy(), 1 + acc, old_len, np.minimum(acc, k - 1)])
        self._rec = rec
        for b in range(B):
            spec = [int(x) for x in ho[3:, b]]
            new = spec[:acc[b]] + [int(rec[b])]
            self.seqs[b].extend(new)
            self.out[b].extend(new)
            new_all.append(new)
        t.n = t.n + 1 + acc
        d.n = old_len + np.minimum(acc, k - 1)
        self.last_accept = acc
        return new_all

    def generate(self, prompts: list[list[int]], max_new: int) -> list[list[int]]:
        self.start(prompts)
        while min(len(o) for o in self.out) < max_new:
            self.step()
        return [o[:max_new] for o in self.out]
