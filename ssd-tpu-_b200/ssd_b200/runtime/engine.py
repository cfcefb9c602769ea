"""LLM inference engine: AR, SD, SSD modes (drop-in for jax_ssd/runtime/engine.py:33-333).

* ``ar``  -- target-only greedy decode (``GreedyDecoder``);
* ``sd``  -- speculative decoding on the device-resident step of
  ``SpeculativeDecoder`` (one greedy prompt: draft k tokens, verify k+1, fused
  acceptance, page rollback, CUDA-graph replay -- the hot path this package
  rebuilds), or ``BatchedSpeculativeDecoder`` when several prompts are given or
  the sampling parameters ask for sampling: the prompts are seated in up to
  ``max(config.batch_buckets)`` rows by the slot ``Scheduler``, and a finished
  row is refilled with the next waiting prompt while the others keep decoding
  (the reference decodes one prompt at a time, engine.py:110-125);
* ``ssd`` -- the async protocol of the reference (``DraftWorker`` thread, host
  queues, ``SpecCache`` keyed by [seq_id, accepted, recovery]) with target
  verification through ``GemmaAdapter.verify`` + ``verify_greedy``; the draft
  and its worker run on their own GPU when there is one for them.

The target (and, in ``ar`` / ``sd`` modes, the draft) lives in a rank group
(``runtime.rank_group``): on one GPU a ``RankState`` in this process; with
``config.tensor_parallel_size = T > 1``, one worker process per GPU 0..T-1,
each holding its weight shards and issuing the same launches (the O / down
all-reduces and the LM-head all-gather are fused into the projection kernels
over NVLink).  In ``ssd`` mode the draft runs unsharded in this process on
``config.draft_device``, by default GPU T -- the reference's target/draft
device split (connect/mesh_allocator.py:47-61).

Greedy decoding is the default, as in the reference (whose sd/ssd paths never
read ``SamplingParams.temperature``, engine.py:235,292); here a temperature > 0
selects rejection sampling on the batched path.  Outputs are truncated to
``max_new_tokens``.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from typing import Iterator

import torch

from .._lib import SSD_MAX_TP
from ..algorithm.async_protocol import DraftCommand, DraftRequest
from ..config import DecodeMode, SSDConfig
from ..kernels.ops import max_tokens_per_forward
from ..models.gemma import PRESETS
from ..models.gemma_adapter import GemmaAdapter
from ..models.model_loader import default_preset, load_weights
from ..sampling_params import SamplingParams
from .metrics import MetricsCollector, RunMetrics, StepMetrics
from .rank_group import LocalRank, RankGroup
from .scheduler import Scheduler
from .sequence import Sequence
from .workers import DraftWorker

TokenCallback = Callable[[int, str], None]


class LLMEngine:
    def __init__(self, config: SSDConfig) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 verify path needs a CUDA device (there is no CPU implementation)")
        self.config = config
        T = int(config.tensor_parallel_size)
        ngpu = torch.cuda.device_count()
        if not 1 <= T <= min(ngpu, SSD_MAX_TP):
            raise ValueError(f"tensor_parallel_size {T} needs 1..{min(ngpu, SSD_MAX_TP)} GPUs (this host has {ngpu})")
        self.tp = T
        mode = config.mode
        self.async_draft = mode in (DecodeMode.SSD, DecodeMode.INSTANCE)
        if config.draft_device:
            self.draft_device = torch.device(config.draft_device)
        elif self.async_draft and T > 1 and ngpu > T:
            self.draft_device = torch.device("cuda", T)  # its own GPU, after the target group
        else:
            self.draft_device = torch.device("cuda", 0)
        tpath, dpath = config.target_model_path, config.draft_model_path
        same = dpath is not None and dpath == tpath
        self._draft_seed = config.seed if same else config.seed + 1
        use_toy = config.use_toy_model
        self.target_preset = tpath if tpath in PRESETS else default_preset("target", use_toy)
        cfg = {"target_model_path": tpath, "draft_model_path": dpath, "use_toy_model": use_toy,
               "seed": config.seed, "draft_seed": self._draft_seed, "max_model_len": config.max_model_len,
               "local_draft": mode != DecodeMode.AR and not self.async_draft, "target_adapter": self.async_draft}
        self.ranks = LocalRank(cfg, 0) if T == 1 else RankGroup(list(range(T)), cfg)
        self.vocab_size = PRESETS[self.target_preset].vocab
        self.draft: GemmaAdapter | None = None
        self.draft_worker: DraftWorker | None = None
        if self.async_draft:
            # the draft adapter and its worker live on the draft's GPU; only token ids cross between GPUs
            dw = load_weights(dpath, use_toy=use_toy, seed=self._draft_seed, role="draft", device=self.draft_device)
            with torch.cuda.device(self.draft_device):
                self.draft = GemmaAdapter(dw, max_model_len=config.max_model_len, name="draft",
                                          max_branches=max(1, config.mq_len))
                self.draft_worker = DraftWorker(config, self.draft)
                self.draft_worker.start()

    # ------------------------------------------------------------ text (byte-level stand-in tokenizer)
    def tokenize(self, text: str) -> list[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")]

    def decode_tokens_to_str(self, token_ids: list[int]) -> str:
        return " ".join(f"t{int(t)}" for t in token_ids)

    # ------------------------------------------------------------ public
    def generate(self, prompts: list[list[int]], sampling: SamplingParams, *,
                 on_token: TokenCallback | None = None) -> tuple[list[list[int]], RunMetrics]:
        collector = MetricsCollector(mode=self.config.mode.value)
        collector.start()
        mode = self.config.mode
        batched = mode == DecodeMode.SD and (len(prompts) > 1 or sampling.temperature > 0)
        # the batched decoder's rows are the slots; the other paths take one prompt at a time
        sched = Scheduler(num_slots=self._num_slots(len(prompts)) if batched else 1)
        seqs = [sched.add_request(p) for p in prompts]
        self.ranks.call("begin")
        try:
            if batched:
                self._run_batched(sched, sampling, on_token, collector)
            else:
                for _ in seqs:
                    (slot, seq), = sched.admit()
                    if mode == DecodeMode.SD:
                        self._run_sd(seq, sampling, on_token, collector)
                    elif self.async_draft:
                        self._run_ssd(seq, sampling, on_token, collector)
                    else:
                        self._run_ar(seq, sampling, on_token, collector)
                    sched.retire(slot)
        finally:
            status = self.ranks.call("end")
        if any(status):
            # a collective whose peer never arrived ends with a timeout status instead of hanging
            raise RuntimeError(f"tensor-parallel collective timed out (rank statuses {status})")
        return [s.completion_token_ids for s in seqs], collector.finish()

    def generate_stream(self, prompt: list[int], sampling: SamplingParams,
                        on_token: TokenCallback | None = None) -> Iterator[tuple[int, str]]:
        collected: list[int] = []

        def _cb(tok: int, s: str) -> None:
            collected.append(tok)
            if on_token:
                on_token(tok, s)

        self.generate([prompt], sampling, on_token=_cb)
        for tok in collected:
            yield tok, self.decode_tokens_to_str([tok])

    def shutdown(self) -> None:
        if self.draft_worker:
            self.draft_worker.stop()
            self.draft_worker = None
        if self.ranks is not None:
            self.ranks.close()
            self.ranks = None

    # ------------------------------------------------------------ modes
    def _num_slots(self, n: int) -> int:
        """Rows of the batched decoder: every prompt, at most max(batch_buckets), and B*(k+1)
        within one forward."""
        dtype = torch.float32 if self.target_preset.startswith("toy") else torch.bfloat16
        cap = max_tokens_per_forward(dtype) // (self.config.speculate_k + 1)
        return max(1, min(n, max(self.config.batch_buckets), cap))

    def _emit(self, seq: Sequence, toks: list[int], limit: int, on_token) -> int:
        n = 0
        for t in toks:
            if seq.num_completion_tokens >= limit:
                break
            seq.append_token(t)
            n += 1
            if on_token:
                on_token(t, self.decode_tokens_to_str([t]))
        return n

    def _max_len(self, longest_prompt: int, sampling: SamplingParams) -> int:
        k = self.config.speculate_k
        n = longest_prompt + sampling.max_new_tokens + 2 * (k + 1) + 16
        if n > self.config.max_model_len + 2 * (k + 1) + 16:
            raise ValueError("prompt + max_new_tokens exceeds max_model_len")
        return n

    def _run_ar(self, seq, sampling, on_token, collector) -> None:
        t0 = time.perf_counter()
        max_len = self._max_len(len(seq.prompt_token_ids), sampling)
        out = self.ranks.call("ar_generate", list(seq.prompt_token_ids), sampling.max_new_tokens, max_len,
                              self.config.block_size)[0]
        collector.record_first_token()
        n = self._emit(seq, out, sampling.max_new_tokens, on_token)
        collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000, accepted_tokens=n))

    def _run_sd(self, seq, sampling, on_token, collector) -> None:
        k = self.config.speculate_k
        max_len = self._max_len(len(seq.prompt_token_ids), sampling)
        first = self.ranks.call("sd_start", list(seq.prompt_token_ids), k, max_len, self.config.block_size)[0]
        self._emit(seq, [first], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            new, verify_ms, acc = self.ranks.call("sd_step")[0]
            n = self._emit(seq, new, sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000, accepted_tokens=n,
                                              verify_device_ms=verify_ms))
            collector.record_accepts([acc])

    def _run_batched(self, sched: Scheduler, sampling, on_token, collector) -> None:
        """Continuous batching over the scheduler's slots (see the module docstring)."""
        k = self.config.speculate_k
        max_len = self._max_len(max(len(s.prompt_token_ids) for s in sched.waiting), sampling)
        temp = float(sampling.temperature)
        self.ranks.call("batch_open", sched.num_slots, k, max_len, self.config.block_size, temp,
                        float(sampling.top_p) if temp > 0 else 1.0, self.config.sampler_x, self.config.seed)
        limit = sampling.max_new_tokens
        first_done = False
        while sched.has_work():
            placed = sched.admit()
            if placed:
                firsts = self.ranks.call("batch_admit", [(slot, s.prompt_token_ids) for slot, s in placed])[0]
                for (slot, seq), f in zip(placed, firsts):
                    self._emit(seq, [f], limit, on_token)
                if not first_done:
                    collector.record_first_token()
                    first_done = True
            for slot, seq in sched.slots():
                if seq.is_finished(None, limit):
                    sched.retire(slot)
                    if not sched.waiting:
                        self.ranks.call("batch_park", slot)
            if not sched.slots():
                continue
            t0 = time.perf_counter()
            new, verify_ms, accepts = self.ranks.call("batch_step")[0]
            active = sched.slots()
            emitted = sum(self._emit(seq, new[slot], limit, on_token) for slot, seq in active)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              accepted_tokens=emitted, verify_device_ms=verify_ms,
                                              sequences=len(active)))
            collector.record_accepts(accepts[slot] for slot, _ in active)

    def _run_ssd(self, seq, sampling, on_token, collector) -> None:
        assert self.draft_worker is not None
        recovery = self.ranks.call("target_prefill", list(seq.prompt_token_ids))[0]
        seq.recovery_token = recovery
        self._emit(seq, [recovery], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        acc = 0
        commit: list[int] | None = None
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            key = torch.tensor([[seq.seq_id, acc, recovery]], dtype=torch.int32)
            self.draft_worker.submit(DraftRequest(DraftCommand.SERVE, key, torch.tensor([seq.num_tokens]),
                                                  torch.zeros((1, 1), dtype=torch.int32), torch.zeros(1),
                                                  prefix_tokens=[list(seq.token_ids)]))
            if commit is not None:  # the previous step's commit runs on the target while the draft drafts
                self.ranks.call("target_commit", commit)
            resp = self.draft_worker.get_response()
            t1 = time.perf_counter()
            spec = [int(t) for t in resp.spec_tokens[0].tolist()]
            outcomes = self.ranks.call("target_verify", [recovery] + spec)
            if len({o[:2] for o in outcomes}) != 1:
                raise RuntimeError(f"tensor-parallel ranks disagree on the verify outcome: {outcomes}")
            acc, recovery, verify_ms = outcomes[0]
            commit = spec[:acc] + [recovery]
            n = self._emit(seq, commit, sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              draft_step_ms=(t1 - t0) * 1000, cache_hit=bool(resp.cache_hit[0]),
                                              accepted_tokens=n, verify_device_ms=verify_ms))
            collector.record_accepts([acc])
        if commit is not None:
            self.ranks.call("target_commit", commit)
