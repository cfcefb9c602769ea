"""Greedy speculative decoding of one sequence on the verify-path kernels.

The device work of a step is replayed from a CUDA graph per draft-feed length
(1 or 2 tokens) once that shape has been seen twice (the first run is eager).

Per step (the sd loop of jax_ssd/runtime/engine.py:230-252, with the KV
bookkeeping a real paged cache needs instead of the reference's per-token
re-commit, gemma_adapter.py:145-152):

1. draft: k greedy forwards of the draft model (first one over the committed
   tokens it has not seen — 1, or 2 after a fully accepted step), each followed
   by ``ssd_argmax_rows`` writing the next draft token straight into the verify
   input row on the device;
2. verify: one target forward over ``[recovery] + draft[k]`` (k+1 tokens), which
   also writes their K/V rows into the target's pages;
3. ``ssd_verify_greedy`` -> accepted count and recovery token (device);
4. one device->host read of (accepted, recovery) and the k+1 verify tokens;
5. ``ssd_page_rollback`` on both caches (issued at the start of the next step,
   from host scalars): target keeps old + 1 + accepted tokens, the draft keeps
   what it computed for accepted tokens; surplus pages return to the free lists.

All device work of a step is stream-ordered with no allocation; the only host
synchronisation is step 4.
"""

from __future__ import annotations

import time

import torch

from ..algorithm.verify import argmax_rows
from .._lib import check, lib, ptr, stream_ptr
from ..kernels.kv_cache import KVCacheState
from ..kernels.ops import max_tokens_per_forward
from ..models.gemma import GemmaRunner, GemmaWeights
from ..workspace import workspace
from .page_manager import PageManager


class _Model:
    def __init__(self, weights: GemmaWeights, max_seq_len: int, block_size: int, k: int, comm=None):
        s = weights.shape
        self.w = weights
        self.num_blocks = (max_seq_len + block_size - 1) // block_size + 2
        self.cache = KVCacheState.allocate(s.num_layers, self.num_blocks, block_size, s.num_kv_heads, s.head_dim,
                                           dtype=weights.dtype, device=weights.device)
        self.pm = PageManager(block_size, self.num_blocks, max_seqs=1, device=weights.device)
        self.runner = GemmaRunner(weights, 1, max(k + 1, max_tokens_per_forward(weights.dtype)), max_seq_len,
                                  comm=comm)
        self.chunk = min(64, max_tokens_per_forward(weights.dtype))
        self.n = 0  # tokens in the cache


class SpeculativeDecoder:
    def __init__(self, target: GemmaWeights, draft: GemmaWeights, k: int = 4, max_seq_len: int = 1024,
                 block_size: int = 16, use_graphs: bool = True, timer=None, comm=None):
        """``comm``: tensor-parallel group (``runtime.tensor_parallel.TPComm``); the
        weights are then this rank's shards and every rank runs the same steps."""
        self.k = k
        self.dev = target.device
        self.max_seq_len = max_seq_len
        self.comm = comm
        self.t = _Model(target, max_seq_len, block_size, k, comm)
        self.d = _Model(draft, max_seq_len, block_size, k, comm)
        V = target.shape.vocab
        if draft.shape.vocab != V:
            raise ValueError("target and draft must share the vocabulary")
        dev = self.dev
        self.vt = torch.zeros((1, k + 1), dtype=torch.int32, device=dev)   # [recovery, draft...]
        self.feed = torch.zeros((1, 2), dtype=torch.int32, device=dev)
        buf = comm.alloc if comm is not None else (
            lambda shape, dtype: torch.empty(shape, dtype=dtype, device=dev))
        self.logits_t = buf((1, k + 1, V), torch.float32)  # written by every rank's LM head block
        self.logits_d = buf((1, V), torch.float32)
        self.acc_rec = torch.zeros(2, dtype=torch.int32, device=dev)
        self.mask = torch.empty((1, k + 1), dtype=torch.uint8, device=dev)
        self.host = torch.zeros(2, dtype=torch.int32).pin_memory()
        # host -> device scalars of one step, copied once per step
        self.h_scal = torch.zeros(16 + k, dtype=torch.int32).pin_memory()
        self.d_scal = torch.zeros(16 + k, dtype=torch.int32, device=dev)
        self.h_roll = torch.zeros(8, dtype=torch.int32).pin_memory()
        self.d_roll = torch.zeros(8, dtype=torch.int32, device=dev)
        self.spec_host = torch.zeros(k + 1, dtype=torch.int32).pin_memory()
        self.ws_greedy = workspace(dev, "sd_greedy", lib().ssd_verify_greedy_workspace_size(1, k, V))
        self.ws_argmax = workspace(dev, "sd_argmax", lib().ssd_verify_greedy_workspace_size(1, 0, V))
        self.tokens: list[int] = []
        # external: inside a captured step these become real event-record nodes that can be timed
        self.ev_verify = (torch.cuda.Event(enable_timing=True, external=True),
                          torch.cuda.Event(enable_timing=True, external=True))
        self.use_graphs = use_graphs
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._capture_stream: torch.cuda.Stream | None = None
        self._seen: dict[int, int] = {}
        self._graph_prof = timer  # projection timer bound into the step (eager or captured)
        self.last_verify_ms = 0.0

    # ------------------------------------------------------------------ helpers
    # Host scalars of one step are written into the pinned ``h_scal`` and copied
    # to ``d_scal`` with ONE async copy before the step's launches; rollback
    # scalars use a second copy after the step's synchronisation point, so no
    # pinned slot is rewritten while a copy from it may still be pending.
    def _scal(self, i: int) -> torch.Tensor:
        return self.d_scal[i:i + 1]

    def _prefill(self, m: _Model, prompt: torch.Tensor, want_logits: bool):
        chunk = m.chunk
        n = prompt.shape[1]
        dev = self.dev
        m.pm.allocate_rows(0, 1, torch.zeros(1, dtype=torch.int32, device=dev),
                           torch.tensor([n], dtype=torch.int32, device=dev), None)
        out = None
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            lg = self.logits_d if (c1 == n and want_logits) else None
            slb = torch.tensor([c0], dtype=torch.int32, device=dev)
            m.runner.forward(prompt[:, c0:c1].contiguous(), slb, m.cache.pages, m.pm.tables, lg, last_only=True)
            out = lg
        m.n = n
        return out

    # ------------------------------------------------------------------ API
    def start(self, prompt: list[int]) -> int:
        """Prefill both models; returns the first generated token (target argmax)."""
        p = torch.tensor([prompt], dtype=torch.int32, device=self.dev)
        lg = self._prefill(self.t, p, True)
        argmax_rows(lg, self.vt[0, 0:1])
        self._prefill(self.d, p, False)
        self.host[:1].copy_(self.vt[0, 0:1], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        first = int(self.host[0])
        self.seq = list(prompt) + [first]
        self.tokens = [first]
        # no rollback is pending before the first step: keep both tables as they are
        self._roll = (self.t.n, 0, self.d.n, 0)
        self._rec = first
        return first

    # Host scalar slots (int32), copied to the device once per step:
    #  0 draft tokens cached | 1 draft tokens to reserve | 2-3 draft feed tokens
    #  4 target tokens cached | 5 verify tokens (k+1) | 6-7 target rollback
    #  (num_tokens, accepted) | 8-9 draft rollback | 10 recovery token
    #  16.. draft forward i: tokens cached before it
    def _host_scalars(self, nf: int) -> None:
        k, t, d, h = self.k, self.t, self.d, self.h_scal
        feed = self.seq[d.n:]
        h[0] = d.n
        h[1] = nf + k - 1
        for j, tok in enumerate(feed):
            h[2 + j] = tok
        h[4] = t.n
        h[5] = k + 1
        h[6], h[7], h[8], h[9] = self._roll
        h[10] = self._rec
        h[16] = d.n
        for i in range(1, k):
            h[16 + i] = d.n + nf + i - 1

    def _device_step(self, nf: int, prof=None) -> None:
        """All device work of one step; stream-ordered, no allocation, capturable."""
        k, t, d = self.k, self.t, self.d
        st = torch.cuda.current_stream()
        self.d_scal.copy_(self.h_scal, non_blocking=True)
        # rollback of the previous verify (no-op values before the first step)
        t.pm.rollback_rows(0, 1, self._scal(6), self._scal(7))
        d.pm.rollback_rows(0, 1, self._scal(8), self._scal(9))
        self.vt[0, 0:1].copy_(self.d_scal[10:11])
        # draft: k greedy forwards, tokens written into vt[0, 1..k]
        d.pm.allocate_rows(0, 1, self._scal(0), self._scal(1), None)
        d.runner.forward(self.d_scal[2:2 + nf].view(1, nf), self._scal(16), d.cache.pages, d.pm.tables,
                         self.logits_d, last_only=True)
        argmax_rows(self.logits_d, self.vt[0, 1:2])
        for i in range(1, k):
            d.runner.forward(self.vt[:, i:i + 1], self._scal(16 + i), d.cache.pages, d.pm.tables, self.logits_d,
                             last_only=True)
            argmax_rows(self.logits_d, self.vt[0, i + 1:i + 2])
        # verify: target forward over k+1 tokens + fused greedy acceptance
        self.ev_verify[0].record(st)
        t.pm.allocate_rows(0, 1, self._scal(4), self._scal(5), None)
        t.runner.forward(self.vt, self._scal(4), t.cache.pages, t.pm.tables, self.logits_t, last_only=False,
                         prof=prof)
        check(lib().ssd_verify_greedy(stream_ptr(), ptr(self.logits_t), ptr(self.vt), ptr(self.acc_rec[0:1]),
                                      ptr(self.acc_rec[1:2]), ptr(self.mask), None, ptr(self.ws_greedy),
                                      self.ws_greedy.numel(), 1, k, self.logits_t.shape[2]), "ssd_verify_greedy")
        self.ev_verify[1].record(st)
        self.host.copy_(self.acc_rec, non_blocking=True)
        self.spec_host.copy_(self.vt[0], non_blocking=True)

    def step(self, prof=None) -> list[int]:
        """One draft+verify+accept iteration (rollback of it runs first in the next one)."""
        k, t, d = self.k, self.t, self.d
        nf = len(self.seq) - d.n
        self._host_scalars(nf)
        g = self._graphs.get(nf) if self.use_graphs else None
        if g is not None:
            g.replay()
        elif self.use_graphs and self._seen.get(nf, 0) >= 1:
            # second sighting of this shape: capture (first run was eager, so every
            # lazily created buffer and cached tensor map already exists), then replay
            # capture on this decoder's own stream, thread-local: under a DeviceGroup every GPU's
            # thread captures its own step at the same time
            g = torch.cuda.CUDAGraph()
            if self._capture_stream is None:
                self._capture_stream = torch.cuda.Stream(device=self.dev)
            with torch.cuda.graph(g, stream=self._capture_stream, capture_error_mode="thread_local"):
                self._device_step(nf, prof=self._graph_prof)
            self._graphs[nf] = g
            g.replay()
        else:
            self._seen[nf] = self._seen.get(nf, 0) + 1
            self._device_step(nf, prof=self._graph_prof if self.use_graphs else prof)
        torch.cuda.current_stream().synchronize()
        if self._graph_prof is not None:
            self._graph_prof.read()
        acc, rec = int(self.host[0]), int(self.host[1])
        spec = [int(x) for x in self.spec_host[1:].tolist()]
        new = spec[:acc] + [rec]
        n_seq_old = len(self.seq)
        self._roll = (t.n, 1 + acc, n_seq_old, min(acc, k - 1))
        self._rec = rec
        t.n = t.n + 1 + acc
        d.n = n_seq_old + min(acc, k - 1)
        self.seq.extend(new)
        self.tokens.extend(new)
        self.last_accept = acc
        self.last_verify_ms = self.ev_verify[0].elapsed_time(self.ev_verify[1])
        return new

    def generate(self, prompt: list[int], max_new: int) -> tuple[list[int], dict]:
        t0 = time.perf_counter()
        self.start(prompt)
        steps = 0
        acc_total = 0
        while len(self.tokens) < max_new:
            self.step()
            steps += 1
            acc_total += self.last_accept
        torch.cuda.current_stream().synchronize()
        return self.tokens[:max_new], {"steps": steps, "accepted": acc_total,
                                       "seconds": time.perf_counter() - t0}


class GreedyDecoder:
    """Target-only greedy decode (the AR loop of engine.py:162-211) on the same kernels."""

    def __init__(self, target: GemmaWeights, max_seq_len: int = 1024, block_size: int = 16, comm=None):
        self.t = _Model(target, max_seq_len, block_size, 1, comm)
        self.dev = target.device
        V = target.shape.vocab
        self.lg = comm.alloc((1, V), torch.float32) if comm is not None else torch.empty(
            (1, V), dtype=torch.float32, device=self.dev)

    def generate(self, prompt: list[int], max_new: int) -> list[int]:
        t, dev, lg = self.t, self.dev, self.lg
        n = len(prompt)
        p = torch.tensor([prompt], dtype=torch.int32, device=dev)
        chunk = t.chunk
        t.pm.allocate_rows(0, 1, torch.zeros(1, dtype=torch.int32, device=dev),
                           torch.tensor([n], dtype=torch.int32, device=dev), None)
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            slb = torch.tensor([c0], dtype=torch.int32, device=dev)
            t.runner.forward(p[:, c0:c1].contiguous(), slb, t.cache.pages, t.pm.tables, lg if c1 == n else None,
                             last_only=True)
        t.n = n
        tok = torch.empty((1, 1), dtype=torch.int32, device=dev)
        argmax_rows(lg, tok[0])
        host = torch.zeros(1, dtype=torch.int32).pin_memory()
        host.copy_(tok[0], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        out = [int(host[0])]
        one = torch.ones(1, dtype=torch.int32, device=dev)
        while len(out) < max_new:
            nn = torch.tensor([t.n], dtype=torch.int32, device=dev)
            t.pm.allocate_rows(0, 1, nn, one, None)
            t.runner.forward(tok, nn, t.cache.pages, t.pm.tables, lg, last_only=True)
            argmax_rows(lg, tok[0])
            host.copy_(tok[0], non_blocking=True)
            torch.cuda.current_stream().synchronize()
            t.n += 1
            out.append(int(host[0]))
        return out
