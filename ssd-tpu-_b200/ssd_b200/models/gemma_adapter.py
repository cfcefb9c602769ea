"""Gemma adapter on the verify-path kernels (replaces jax_ssd/models/gemma_adapter.py).

Implements the ``DecodeModelAdapter`` protocol (jax_ssd/models/base.py:34-60)
and the duck-typed extras the reference engine calls (``allocate_kv``,
``commit_tokens``, ``draft_speculate``, ``tokenize``, ``decode_tokens_to_str``),
with a real paged KV cache instead of the reference's dummy one:

* ``verify`` runs one ``ssd_gemma_forward`` over the k+1 tokens at their true
  positions (the reference passes ``arange(k+1)``, engine.py:234, and its
  adapter ignores it) and writes their K/V rows;
* ``commit_tokens(accepted + [recovery])`` keeps the verified recovery token and
  the accepted drafts in the cache and rolls the rest back (``ssd_page_rollback``)
  -- the reference instead re-runs one forward per committed token
  (gemma_adapter.py:145-152);
* ``draft_speculate(prefix, k)`` reuses the draft cache up to the longest
  common prefix with what it already holds, feeds the remaining tokens, then
  drafts k greedy tokens (the reference re-prefills the whole prefix each time
  and drops its first prediction, gemma_adapter.py:154-175).
"""

from __future__ import annotations

import time
from typing import Callable

import torch

from ..algorithm.verify import argmax_rows
from ..kernels.kv_cache import KVCacheState
from ..kernels.ops import max_tokens_per_forward
from ..runtime.page_manager import PageManager
from .base import DecodeResult, PrefillResult, VerifyResultModel
from .gemma import GemmaRunner, GemmaWeights


class GemmaAdapter:
    def __init__(self, model_path: GemmaWeights | str | None = None, vocab_size: int | None = None,
                 share_key: str | None = None, mesh=None, devices=None, role: str = "target", *,
                 max_model_len: int = 4096, block_size: int = 16, max_tokens: int = 64, name: str | None = None,
                 max_branches: int = 0, comm=None) -> None:
        """Positional arguments in the reference's order (gemma_adapter.py:28-36).

        ``model_path``: a ``GemmaWeights`` already on the device, or a model path.  A path names a
        random-init preset (``models.model_loader.load_weights``: a preset name, else the role's
        default preset, the toy pair when ``SSD_USE_TOY_MODEL`` is set).  ``vocab_size``,
        ``share_key``, ``mesh`` and ``devices`` place the reference's JAX arrays and have no effect
        here (the vocabulary comes from the weights, as the reference takes it from the model
        config).  Everything this adapter adds is keyword-only.

        ``comm`` (a ``runtime.tensor_parallel.TPComm``): the weights are one rank's shard and
        every rank of the group makes the same calls; logits land in the group's symmetric heap
        (the LM head all-gathers into it) and are returned as copies."""
        if isinstance(model_path, GemmaWeights):
            weights = model_path
        else:
            from ..config import _env_bool
            from .model_loader import load_weights

            weights = load_weights(model_path, use_toy=_env_bool("SSD_USE_TOY_MODEL"), role=role)
        name = name or role
        s = weights.shape
        self.w = weights
        self.name = name
        self.vocab_size = s.vocab
        self.max_model_len = max_model_len
        self.block_size = block_size
        self.max_branches = int(max_branches)
        per_seq = (max_model_len + block_size - 1) // block_size + 2
        # row 0 holds the sequence; rows 1.. are branch rows forked from it (shared trunk pages
        # plus one private block each for the partial trunk page and the branch tokens)
        self.num_blocks = per_seq + self.max_branches * 4
        self.dev = weights.device
        self.chunk = min(64, max_tokens_per_forward(weights.dtype))
        self.comm = comm
        self.runner = GemmaRunner(weights, 1 + self.max_branches, max(self.chunk, max_tokens), max_model_len,
                                  comm=comm)
        self.cache = KVCacheState.allocate(s.num_layers, self.num_blocks, block_size, s.num_kv_heads, s.head_dim,
                                           dtype=weights.dtype, device=self.dev)
        self.pm = PageManager(block_size, self.num_blocks, max_seqs=1 + self.max_branches,
                              max_blocks_per_seq=per_seq, device=self.dev)
        self.cached: list[int] = []   # tokens whose K/V rows are valid in the cache
        self.pending: list[int] = []  # tokens of the last verify (written, not yet committed)
        # logits rows of one forward: a symmetric heap buffer under tensor parallelism
        self._lg_rows = max(self.chunk, max_tokens, 1 + self.max_branches)
        self._lg_heap = comm.alloc((self._lg_rows, s.vocab), torch.float32) if comm is not None else None
        self._lg1 = self._logits(1)
        self._h_scal = self._d_scal = self._d_tok = None  # draft_speculate's scalars and tokens
        self._scal_ev: torch.cuda.Event | None = None

    def _logits(self, rows: int) -> torch.Tensor:
        """A [rows, V] fp32 buffer the forward may write its logits into."""
        if self._lg_heap is None:
            return torch.empty((rows, self.vocab_size), dtype=torch.float32, device=self.dev)
        if rows > self._lg_rows:
            raise ValueError(f"{rows} logits rows exceed the adapter's {self._lg_rows}")
        return self._lg_heap[:rows]

    # ------------------------------------------------------------ cache state
    def _i32(self, v) -> torch.Tensor:
        return torch.tensor([int(v)], dtype=torch.int32, device=self.dev)

    def _truncate(self, n: int) -> None:
        """Keep the first n cached tokens; surplus pages go back to the free list."""
        if n < len(self.cached) or self.pending:
            self.pm.rollback_rows(0, 1, self._i32(n), self._i32(0))
        self.cached = self.cached[:n]
        self.pending = []

    def _run(self, tokens: list[int], logits: torch.Tensor | None, last_only: bool) -> torch.Tensor | None:
        """Append `tokens` to the cache (chunked); returns the logits of the last chunk."""
        n0 = len(self.cached)
        if n0 + len(tokens) > self.max_model_len:
            raise ValueError("sequence exceeds max_model_len")
        self.pm.allocate_rows(0, 1, self._i32(n0), self._i32(len(tokens)), None)
        out = None
        for c0 in range(0, len(tokens), self.chunk):
            part = tokens[c0:c0 + self.chunk]
            last = c0 + self.chunk >= len(tokens)
            t = torch.tensor([part], dtype=torch.int32, device=self.dev)
            lg = logits if last else None
            self.runner.forward(t, self._i32(n0 + c0), self.cache.pages, self.pm.tables, lg, last_only=last_only)
            out = lg
        self.cached.extend(int(x) for x in tokens)
        return out

    def reset_cache(self) -> None:
        """Forget the cached tokens and release their pages (gemma_adapter.py:74-75)."""
        self._truncate(0)

    def allocate_kv(self) -> KVCacheState:
        self.reset_cache()
        return self.cache

    # ------------------------------------------------------------ protocol
    def prefill(self, token_ids, kv_cache=None, page_table=None) -> PrefillResult:
        self._truncate(0)
        toks = [int(x) for x in torch.as_tensor(token_ids).reshape(-1).tolist()]
        lg = self._run(toks, self._lg1, last_only=True)
        return PrefillResult(logits=lg.clone(), kv_cache=self.cache)

    def decode(self, token_id: int, position: int | None = None, kv_cache=None, page_table=None) -> DecodeResult:
        if self.pending:
            self._truncate(len(self.cached))
        lg = self._run([int(token_id)], self._lg1, last_only=True)
        nxt = torch.empty(1, dtype=torch.int32, device=self.dev)
        argmax_rows(lg, nxt)
        return DecodeResult(logits=lg.clone(), kv_cache=self.cache, next_token=int(nxt.item()))

    def verify(self, token_ids_kp1, positions=None, kv_cache=None, page_table=None) -> VerifyResultModel:
        if self.pending:
            self._truncate(len(self.cached))
        toks = [int(x) for x in torch.as_tensor(token_ids_kp1).reshape(-1).tolist()]
        lg = self._logits(len(toks)).view(1, len(toks), self.vocab_size)
        n0 = len(self.cached)
        self.pm.allocate_rows(0, 1, self._i32(n0), self._i32(len(toks)), None)
        self.runner.forward(torch.tensor([toks], dtype=torch.int32, device=self.dev), self._i32(n0),
                            self.cache.pages, self.pm.tables, lg, last_only=False)
        self.pending = toks
        return VerifyResultModel(logits=lg if self.comm is None else lg.clone(), kv_cache=self.cache)

    def commit_tokens(self, token_ids: list[int]) -> None:
        """After verify([r] + draft): token_ids = accepted + [new recovery] keeps r + accepted."""
        if self.pending:
            keep = min(len(token_ids), len(self.pending))  # r and the len(token_ids) - 1 accepted drafts
            n = len(self.cached) + keep
            self.cached.extend(self.pending[:keep])
            self.pending = []
            self.pm.rollback_rows(0, 1, self._i32(n), self._i32(0))
        # tokens that were never verified (e.g. a fresh recovery) enter with the next forward

    def draft_speculate(self, prefix_tokens: list[int], k: int, *,
                        with_bonus: bool = False) -> tuple[list[int], torch.Tensor]:
        """k greedy draft tokens after `prefix_tokens` and the logits that chose them, [k, V]
        (``with_bonus``: one more forward over the last draft, logits [k+1, V])."""
        prefix = [int(t) for t in prefix_tokens]
        common = 0
        for a, b in zip(self.cached, prefix):
            if a != b:
                break
            common += 1
        common = min(common, len(prefix) - 1)  # always feed at least one token
        rows = k + 1 if with_bonus else k
        if 1 <= rows and len(prefix) - common <= self.chunk and self.comm is None:
            return self._draft_chained(prefix, common, k, rows)
        self._truncate(common)
        logits = torch.empty((rows, self.vocab_size), dtype=torch.float32, device=self.dev)
        feed = prefix[common:]
        spec: list[int] = []
        nxt = torch.empty(1, dtype=torch.int32, device=self.dev)
        for i in range(rows):
            lg = self._run(feed, self._lg1, last_only=True)
            logits[i].copy_(lg[0])
            if i == k:
                break
            argmax_rows(lg, nxt)
            spec.append(int(nxt.item()))
            feed = [spec[-1]]
        return spec, logits

    def _draft_chained(self, prefix: list[int], common: int, k: int, rows: int) -> tuple[list[int], torch.Tensor]:
        """``draft_speculate`` for a feed of at most one chunk, with the same forwards, tokens and
        positions, but each draft token goes from its argmax straight into the next forward on the
        device: the call's scalars (rollback, page allocation, positions, feed tokens) reach the
        device in one copy from pinned memory and the k tokens come back in one copy, instead of a
        few blocking copies per token."""
        feed = prefix[common:]
        f = len(feed)
        if common + f + rows - 1 > self.max_model_len:
            raise ValueError("sequence exceeds max_model_len")
        # [truncate-to, 0, tokens before the feed, tokens to allocate, positions of forwards 1.., feed]
        vals = [common, 0, common, f + rows - 1] + [common + f + i - 1 for i in range(1, rows)] + feed
        n = len(vals)
        if self._scal_ev is not None:
            self._scal_ev.synchronize()  # the previous call's upload has left the pinned buffer
        if self._h_scal is None or self._h_scal.numel() < n:
            self._h_scal = torch.empty(max(256, n), dtype=torch.int32, pin_memory=True)
            self._d_scal = torch.empty(max(256, n), dtype=torch.int32, device=self.dev)
            self._d_tok = torch.empty(max(256, n), dtype=torch.int32, device=self.dev)
            self._scal_ev = torch.cuda.Event()
        self._h_scal[:n] = torch.tensor(vals, dtype=torch.int32)
        d = self._d_scal
        d[:n].copy_(self._h_scal[:n], non_blocking=True)
        self._scal_ev.record()
        if common < len(self.cached) or self.pending:
            self.pm.rollback_rows(0, 1, d[0:1], d[1:2])
        self.cached = self.cached[:common]
        self.pending = []
        self.pm.allocate_rows(0, 1, d[2:3], d[3:4], None)
        logits = torch.empty((rows, self.vocab_size), dtype=torch.float32, device=self.dev)
        toks = self._d_tok
        lg = self._lg1
        pos0 = 4 + rows - 1
        self.runner.forward(d[pos0:pos0 + f].view(1, f), d[2:3], self.cache.pages, self.pm.tables, lg,
                            last_only=True)
        logits[0].copy_(lg[0])
        if k > 0:
            argmax_rows(lg, toks[0:1])
        for i in range(1, rows):
            self.runner.forward(toks[i - 1:i].view(1, 1), d[4 + i - 1:4 + i], self.cache.pages, self.pm.tables, lg,
                                last_only=True)
            logits[i].copy_(lg[0])
            if i < k:
                argmax_rows(lg, toks[i:i + 1])
        spec = [int(t) for t in toks[:k].cpu().tolist()] if k > 0 else []
        self.cached = prefix[:common] + feed + spec[:rows - 1]
        return spec, logits

    def draft_branches(self, prefix_tokens: list[int], feeds: list[list[int]], k: int,
                       stop: Callable[[], bool] | None = None) -> list[list[int]]:
        """k greedy draft tokens for each branch ``prefix + feeds[i]``, all branches at once.

        Row 0 is brought to hold exactly the prefix (common-prefix reuse, as in
        ``draft_speculate``); branch rows are forked from it (``ssd_page_fork``: trunk
        pages shared, the partial page copied), then one forward over every branch's
        feed (ragged) and k-1 one-token forwards run over all branch rows, and the
        branch rows are released.  Each branch's tokens equal
        ``draft_speculate(prefix + feeds[i], k)[0]`` (batch invariance); branch
        attention is the paged attention over the forked tables.

        ``stop``: polled while each forward runs (the host then issues one forward
        at a time); once it returns True no further forward is issued, the branch
        rows are released and the branches finished so far are returned (a
        prefix of ``feeds``' order, possibly shorter than ``feeds``).
        """
        prefix = [int(t) for t in prefix_tokens]
        n_all = len(feeds)
        if n_all == 0:
            return []
        if self.max_branches <= 0 or any(len(f) == 0 for f in feeds):
            return [self.draft_speculate(prefix + list(f), k)[0] for f in feeds]
        common = 0
        for a, b in zip(self.cached, prefix):
            if a != b:
                break
            common += 1
        self._truncate(common)
        if len(prefix) > common:
            self._run(prefix[common:], None, last_only=True)
        n0 = len(prefix)
        out: list[list[int]] = []
        cap = max_tokens_per_forward(self.w.dtype)
        tmax = max(len(f) for f in feeds)
        group = max(1, min(self.max_branches, cap // max(tmax, 1)))
        for g0 in range(0, n_all, group):
            fs = [list(f) for f in feeds[g0:g0 + group]]
            n = len(fs)
            ok = self.pm.fork_rows(0, 1, n, n0, self.cache)
            if not bool(ok.all()):
                self.pm.free_rows(1, n)
                out.extend(self.draft_speculate(prefix + f, k)[0] for f in fs)
                continue
            ql = [len(f) for f in fs]
            t = max(ql)
            toks = torch.zeros((n, t), dtype=torch.int32)
            for i, f in enumerate(fs):
                toks[i, :len(f)] = torch.tensor(f, dtype=torch.int32)
            toks = toks.to(self.dev)
            qlen = torch.tensor(ql, dtype=torch.int32, device=self.dev)
            base = torch.full((n,), n0, dtype=torch.int32, device=self.dev)
            self.pm.allocate_rows(1, n, base, qlen + (k - 1), None)
            lg = self._logits(n)
            nxt = torch.empty((k, n), dtype=torch.int32, device=self.dev)
            tables = self.pm.tables[1:1 + n]
            self.runner.forward(toks, base, self.cache.pages, tables, lg, q_lens=qlen, last_only=True)
            argmax_rows(lg, nxt[0])
            stopped = False
            for i in range(1, k):
                if stop is not None and self._wait_or_stop(stop):
                    stopped = True
                    break
                self.runner.forward(nxt[i - 1].view(n, 1), base + qlen + (i - 1), self.cache.pages, tables, lg,
                                    last_only=True)
                argmax_rows(lg, nxt[i])
            self.pm.free_rows(1, n)
            if stopped:
                break
            host = nxt.t().cpu().tolist()
            out.extend([int(x) for x in row] for row in host)
        return out

    def _wait_or_stop(self, stop: Callable[[], bool]) -> bool:
        """Wait for the work issued so far, polling ``stop``; True as soon as it returns True."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        while not ev.query():
            if stop():
                return True
            time.sleep(50e-6)
        return stop()

    def tokenize(self, text: str) -> list[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")]

    def decode_tokens_to_str(self, token_ids: list[int]) -> str:
        return " ".join(f"t{int(t)}" for t in token_ids)
