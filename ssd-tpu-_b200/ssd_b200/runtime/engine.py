"""LLM inference engine: AR, SD, SSD modes (drop-in for jax_ssd/runtime/engine.py:33-333).

* ``ar``  -- target-only greedy decode (``GreedyDecoder``);
* ``sd``  -- speculative decoding on the device-resident step of
  ``SpeculativeDecoder`` (one greedy prompt: draft k tokens, verify k+1, fused
  acceptance, page rollback, CUDA-graph replay -- the hot path this package
  rebuilds), or ``BatchedSpeculativeDecoder`` when several prompts are given or
  the sampling parameters ask for sampling: the prompts are seated in up to
  ``max(config.batch_buckets)`` rows by the slot ``Scheduler``, a finished row
  is refilled with the next waiting prompt while the others keep decoding
  (the reference decodes one prompt at a time, engine.py:110-125);
* ``ssd`` -- the async protocol of the reference (``DraftWorker`` thread, host
  queues, ``SpecCache`` keyed by [seq_id, accepted, recovery]) with target
  verification through ``GemmaAdapter.verify`` + ``verify_greedy``; the draft
  and its worker run on their own GPU when there is one for them.

Tensor parallelism (``config.tensor_parallel_size = T > 1``): the target is
sharded over GPUs 0..T-1, each driven by its own thread of a ``DeviceGroup``
(every rank issues the same launches; the O / down all-reduces and the LM-head
all-gather are fused into the projection kernels over NVLink peer memory).  In
``ar`` and ``sd`` modes the draft is sharded over the same GPUs; in ``ssd`` mode
it runs unsharded on ``config.draft_device``, by default GPU T -- the
reference's target/draft device split (connect/mesh_allocator.py:47-61).

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
from ..algorithm.verify import verify_greedy
from ..config import DecodeMode, SSDConfig
from ..kernels.ops import max_tokens_per_forward
from ..models.gemma import PRESETS
from ..models.gemma_adapter import GemmaAdapter
from ..models.model_loader import default_preset, load_sharded_weights, load_weights
from ..sampling_params import SamplingParams
from .batched import BatchedSpeculativeDecoder
from .device_group import DeviceGroup
from .metrics import MetricsCollector, RunMetrics, StepMetrics
from .scheduler import Scheduler
from .sequence import Sequence
from .speculative import GreedyDecoder, SpeculativeDecoder
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
        self.target_devices = [torch.device("cuda", i) for i in range(T)]
        mode = config.mode
        self.async_draft = mode in (DecodeMode.SSD, DecodeMode.INSTANCE)
        if config.draft_device:
            self.draft_device = torch.device(config.draft_device)
        elif self.async_draft and T > 1 and ngpu > T:
            self.draft_device = torch.device("cuda", T)  # its own GPU, after the target group
        else:
            self.draft_device = self.target_devices[0]
        self.sharded_draft = T > 1 and not self.async_draft
        self.group = DeviceGroup(self.target_devices) if T > 1 else None
        self.comms = None
        tpath = config.target_model_path
        dpath = config.draft_model_path
        same = dpath is not None and dpath == tpath
        dseed = config.seed if same else config.seed + 1
        if T == 1:
            self.target_w = [load_weights(tpath, use_toy=config.use_toy_model, seed=config.seed, role="target",
                                          device=self.target_devices[0])]
        else:
            from .tensor_parallel import TPComm

            self.target_w = self._each(lambda r: load_sharded_weights(
                tpath, r, T, use_toy=config.use_toy_model, seed=config.seed, role="target",
                device=self.target_devices[r]))
            d_model = max(PRESETS[self._preset(tpath, "target")].d_model,
                          PRESETS[self._preset(dpath, "draft")].d_model)
            self.comms = TPComm.local_group(self.target_devices, heap_bytes=512 << 20, max_m=256, max_n=d_model)
        self.draft_w = None
        if mode != DecodeMode.AR:
            if self.sharded_draft:
                self.draft_w = self._each(lambda r: load_sharded_weights(
                    dpath, r, T, use_toy=config.use_toy_model, seed=dseed, role="draft",
                    device=self.target_devices[r]))
            else:
                self.draft_w = [load_weights(dpath, use_toy=config.use_toy_model, seed=dseed, role="draft",
                                             device=self.draft_device)]
        # target adapters (prefill / verify / commit_tokens of the ssd loop), one per rank
        self.targets = self._each(lambda r: GemmaAdapter(
            self.target_w[r], max_model_len=config.max_model_len, name="target",
            comm=self.comms[r] if self.comms else None))
        self.target = self.targets[0]
        self.draft: GemmaAdapter | None = None
        self.draft_worker: DraftWorker | None = None
        if self.async_draft:
            # the draft adapter and its worker live on the draft's GPU; only token ids cross between GPUs
            with torch.cuda.device(self.draft_device):
                self.draft = GemmaAdapter(self.draft_w[0], max_model_len=config.max_model_len, name="draft",
                                          max_branches=max(1, config.mq_len))
                self.draft_worker = DraftWorker(config, self.draft)
                self.draft_worker.start()

    # ------------------------------------------------------------ helpers
    def _preset(self, path, role: str) -> str:
        return path if path in PRESETS else default_preset(role, self.config.use_toy_model)

    def _each(self, fn):
        """fn(rank) on every rank of the target group (each on its GPU), results in rank order."""
        if self.group is None:
            with torch.cuda.device(self.target_devices[0]):
                return [fn(0)]
        return self.group.run(fn)

    def _comm(self, r: int):
        return self.comms[r] if self.comms else None

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
        marks = self._each(lambda r: self.comms[r].mark()) if self.comms else None
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
            if marks is not None:  # the decoders' symmetric buffers are free again
                self._each(lambda r: torch.cuda.current_stream().synchronize())
                self._each(lambda r: self.comms[r].release(marks[r]))
        if self.comms:
            # a collective whose peer never arrived ends with a timeout status instead of hanging
            status = self._each(lambda r: self.comms[r].status())
            if any(status):
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
            yield tok, self.target.decode_tokens_to_str([tok])

    def shutdown(self) -> None:
        if self.draft_worker:
            self.draft_worker.stop()
            self.draft_worker = None
        if self.comms:
            # the adapters' logits buffers are views of the heaps: drop them before the heaps go
            self.targets = []
            self.target = None
            import gc

            gc.collect()
            self._each(lambda r: self.comms[r].close())
            self.comms = None
        if self.group is not None:
            self.group.close()
            self.group = None

    # ------------------------------------------------------------ modes
    def _num_slots(self, n: int) -> int:
        """Rows of the batched decoder: every prompt, at most max(batch_buckets), and B*(k+1)
        within one forward."""
        cap = max_tokens_per_forward(self.target_w[0].dtype) // (self.config.speculate_k + 1)
        return max(1, min(n, max(self.config.batch_buckets), cap))

    def _emit(self, seq: Sequence, toks: list[int], limit: int, on_token) -> int:
        n = 0
        for t in toks:
            if seq.num_completion_tokens >= limit:
                break
            seq.append_token(t)
            n += 1
            if on_token:
                on_token(t, self.target.decode_tokens_to_str([t]))
        return n

    def _max_len(self, seq: Sequence, sampling: SamplingParams) -> int:
        k = self.config.speculate_k
        n = len(seq.prompt_token_ids) + sampling.max_new_tokens + 2 * (k + 1) + 16
        if n > self.config.max_model_len + 2 * (k + 1) + 16:
            raise ValueError("prompt + max_new_tokens exceeds max_model_len")
        return n

    def _run_ar(self, seq, sampling, on_token, collector) -> None:
        t0 = time.perf_counter()
        max_len = self._max_len(seq, sampling)
        bs = self.config.block_size
        prompt = list(seq.prompt_token_ids)
        outs = self._each(lambda r: GreedyDecoder(self.target_w[r], max_seq_len=max_len, block_size=bs,
                                                  comm=self._comm(r)).generate(prompt, sampling.max_new_tokens))
        collector.record_first_token()
        n = self._emit(seq, outs[0], sampling.max_new_tokens, on_token)
        collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000, accepted_tokens=n))

    def _run_sd(self, seq, sampling, on_token, collector) -> None:
        k = self.config.speculate_k
        max_len = self._max_len(seq, sampling)
        bs = self.config.block_size
        decs = self._each(lambda r: SpeculativeDecoder(self.target_w[r], self.draft_w[r], k=k, max_seq_len=max_len,
                                                       block_size=bs, comm=self._comm(r)))
        prompt = list(seq.prompt_token_ids)
        first = self._each(lambda r: decs[r].start(prompt))[0]
        self._emit(seq, [first], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            new = self._each(lambda r: decs[r].step())[0]
            n = self._emit(seq, new, sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000, accepted_tokens=n,
                                              verify_device_ms=decs[0].last_verify_ms))
            collector.record_accepts([decs[0].last_accept])

    def _run_batched(self, sched: Scheduler, sampling, on_token, collector) -> None:
        """Continuous batching over the scheduler's slots (see the module docstring)."""
        k = self.config.speculate_k
        B = sched.num_slots
        longest = max(len(s.prompt_token_ids) for s in sched.waiting)
        max_len = longest + sampling.max_new_tokens + 2 * (k + 1) + 16
        if max_len > self.config.max_model_len + 2 * (k + 1) + 16:
            raise ValueError("prompt + max_new_tokens exceeds max_model_len")
        temp = float(sampling.temperature)
        decs = self._each(lambda r: BatchedSpeculativeDecoder(
            self.target_w[r], self.draft_w[r], batch=B, k=k, max_seq_len=max_len, block_size=self.config.block_size,
            temperature=temp, top_p=float(sampling.top_p) if temp > 0 else 1.0, sampler_x=self.config.sampler_x,
            seed=self.config.seed, comm=self._comm(r)))
        limit = sampling.max_new_tokens
        first_done = False
        while sched.has_work():
            placed = sched.admit()
            if placed:
                firsts = self._each(lambda r: [decs[r].admit(slot, seq.prompt_token_ids) for slot, seq in placed])[0]
                for (slot, seq), f in zip(placed, firsts):
                    self._emit(seq, [f], limit, on_token)
                if not first_done:
                    collector.record_first_token()
                    first_done = True
            for slot, seq in sched.slots():
                if seq.is_finished(None, limit):
                    sched.retire(slot)
                    if not sched.waiting:
                        self._each(lambda r: decs[r].park(slot))
            if not sched.slots():
                continue
            t0 = time.perf_counter()
            new = self._each(lambda r: decs[r].step())[0]
            emitted = 0
            active = sched.slots()
            for slot, seq in active:
                emitted += self._emit(seq, new[slot], limit, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              accepted_tokens=emitted, verify_device_ms=decs[0].last_verify_ms,
                                              sequences=len(active)))
            collector.record_accepts(int(decs[0].last_accept[slot]) for slot, _ in active)

    def _run_ssd(self, seq, sampling, on_token, collector) -> None:
        assert self.draft_worker is not None
        prompt = torch.tensor(seq.prompt_token_ids, dtype=torch.int32)
        pre = self._each(lambda r: self.targets[r].prefill(prompt))[0]
        recovery = int(pre.logits[0].argmax().item())
        seq.recovery_token = recovery
        self._emit(seq, [recovery], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        acc = 0
        ev = self._verify_events()
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            key = torch.tensor([[seq.seq_id, acc, recovery]], dtype=torch.int32)
            self.draft_worker.submit(DraftRequest(DraftCommand.SERVE, key, torch.tensor([seq.num_tokens]),
                                                  torch.zeros((1, 1), dtype=torch.int32), torch.zeros(1),
                                                  prefix_tokens=[list(seq.token_ids)]))
            resp = self.draft_worker.get_response()
            t1 = time.perf_counter()
            spec = [int(t) for t in resp.spec_tokens[0].tolist()]
            spec_kp1 = [recovery] + spec

            def verify(r):
                st = torch.cuda.current_stream()
                if r == 0:
                    ev[0].record(st)
                vres = self.targets[r].verify(torch.tensor([spec_kp1], dtype=torch.int32))
                vout = verify_greedy(vres.logits, torch.tensor([spec_kp1], dtype=torch.int32, device=vres.logits.device))
                if r == 0:
                    ev[1].record(st)
                return int(vout.accept_until[0]), int(vout.recovery_tokens[0])

            outcomes = self._each(verify)
            if len(set(outcomes)) != 1:
                raise RuntimeError(f"tensor-parallel ranks disagree on the verify outcome: {outcomes}")
            acc, recovery = outcomes[0]
            commit = spec[:acc] + [recovery]
            self._each(lambda r: self.targets[r].commit_tokens(commit))
            n = self._emit(seq, commit, sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              draft_step_ms=(t1 - t0) * 1000, cache_hit=bool(resp.cache_hit[0]),
                                              accepted_tokens=n, verify_device_ms=ev[0].elapsed_time(ev[1])))
            collector.record_accepts([acc])

    def _verify_events(self):
        with torch.cuda.device(self.target_devices[0]):
            return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
