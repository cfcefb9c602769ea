"""LLM inference engine: AR, SD, SSD modes (drop-in for jax_ssd/runtime/engine.py:33-333).

* ``ar``  -- target-only greedy decode (``GreedyDecoder``);
* ``sd``  -- greedy speculative decoding with the device-resident step of
  ``SpeculativeDecoder`` (draft k tokens, verify k+1, fused acceptance, page
  rollback; CUDA-graph replay), the hot path this package rebuilds;
* ``ssd`` -- the async protocol of the reference (``DraftWorker`` thread, host
  queues, ``SpecCache`` keyed by [seq_id, accepted, recovery]) with target
  verification through ``GemmaAdapter.verify`` + ``verify_greedy``.

As in the reference, prompts are decoded one at a time and the engine is
greedy (``SamplingParams.temperature`` is not read on these paths,
engine.py:235,292).  Outputs are truncated to ``max_new_tokens``.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from typing import Iterator

import torch

from ..algorithm.async_protocol import DraftCommand, DraftRequest
from ..algorithm.verify import verify_greedy
from ..config import DecodeMode, SSDConfig
from ..models.gemma_adapter import GemmaAdapter
from ..models.model_loader import load_weights
from ..sampling_params import SamplingParams
from .metrics import MetricsCollector, RunMetrics, StepMetrics
from .page_manager import PageManager
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
        self.page_manager = PageManager(block_size=config.block_size, num_blocks=config.num_blocks)
        self.scheduler = Scheduler(config, self.page_manager)
        self.target_w = load_weights(config.target_model_path, use_toy=config.use_toy_model,
                                     seed=config.seed, role="target")
        self.draft_w = None
        self.draft_worker: DraftWorker | None = None
        self.target = GemmaAdapter(self.target_w, max_model_len=config.max_model_len, name="target")
        self.draft: GemmaAdapter | None = None
        if config.mode != DecodeMode.AR:
            same = config.draft_model_path is not None and config.draft_model_path == config.target_model_path
            async_draft = config.mode in (DecodeMode.SSD, DecodeMode.INSTANCE)
            ddev = torch.device(config.draft_device) if (async_draft and config.draft_device) else \
                torch.device("cuda", torch.cuda.current_device())
            self.draft_w = load_weights(config.draft_model_path, use_toy=config.use_toy_model,
                                        seed=config.seed if same else config.seed + 1, role="draft", device=ddev)
        if config.mode in (DecodeMode.SSD, DecodeMode.INSTANCE):
            # the draft adapter and its worker live on the draft's GPU (its own GPU when
            # config.draft_device names one); only token ids cross between the GPUs
            with torch.cuda.device(self.draft_w.device):
                self.draft = GemmaAdapter(self.draft_w, max_model_len=config.max_model_len, name="draft",
                                          max_branches=max(1, config.mq_len))
                self.draft_worker = DraftWorker(config, self.draft)
                self.draft_worker.start()

    # ------------------------------------------------------------ public
    def generate(self, prompts: list[list[int]], sampling: SamplingParams, *,
                 on_token: TokenCallback | None = None) -> tuple[list[list[int]], RunMetrics]:
        collector = MetricsCollector(mode=self.config.mode.value)
        collector.start()
        outputs: list[list[int]] = []
        for prompt in prompts:
            seq = self.scheduler.add_request(prompt)
            self.scheduler.schedule()
            if self.config.mode == DecodeMode.SD:
                tokens = self._run_sd(seq, sampling, on_token, collector)
            elif self.config.mode in (DecodeMode.SSD, DecodeMode.INSTANCE):
                tokens = self._run_ssd(seq, sampling, on_token, collector)
            else:
                tokens = self._run_ar(seq, sampling, on_token, collector)
            outputs.append(tokens)
            if seq in self.scheduler.running:
                self.scheduler._finish(seq)
        return outputs, collector.finish()

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

    # ------------------------------------------------------------ modes
    def _emit(self, seq: Sequence, toks: list[int], limit: int, on_token) -> None:
        for t in toks:
            if seq.num_completion_tokens >= limit:
                break
            seq.append_token(t)
            if on_token:
                on_token(t, self.target.decode_tokens_to_str([t]))

    def _max_len(self, seq: Sequence, sampling: SamplingParams) -> int:
        k = self.config.speculate_k
        n = len(seq.prompt_token_ids) + sampling.max_new_tokens + 2 * (k + 1) + 16
        if n > self.config.max_model_len + 2 * (k + 1) + 16:
            raise ValueError("prompt + max_new_tokens exceeds max_model_len")
        return n

    def _run_ar(self, seq, sampling, on_token, collector) -> list[int]:
        t0 = time.perf_counter()
        dec = GreedyDecoder(self.target_w, max_seq_len=self._max_len(seq, sampling), block_size=self.config.block_size)
        out = dec.generate(list(seq.prompt_token_ids), sampling.max_new_tokens)
        collector.record_first_token()
        self._emit(seq, out, sampling.max_new_tokens, on_token)
        collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                          accepted_tokens=len(out)))
        return seq.completion_token_ids

    def _run_sd(self, seq, sampling, on_token, collector) -> list[int]:
        k = self.config.speculate_k
        dec = SpeculativeDecoder(self.target_w, self.draft_w, k=k, max_seq_len=self._max_len(seq, sampling),
                                 block_size=self.config.block_size)
        first = dec.start(list(seq.prompt_token_ids))
        self._emit(seq, [first], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            new = dec.step()
            self._emit(seq, new, sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              accepted_tokens=len(new), verify_device_ms=dec.last_verify_ms))
        return seq.completion_token_ids

    def _run_ssd(self, seq, sampling, on_token, collector) -> list[int]:
        assert self.draft_worker is not None
        k = self.config.speculate_k
        pre = self.target.prefill(torch.tensor(seq.prompt_token_ids, dtype=torch.int32))
        recovery = int(pre.logits[0].argmax().item())
        seq.recovery_token = recovery
        self._emit(seq, [recovery], sampling.max_new_tokens, on_token)
        collector.record_first_token()
        acc = 0
        while not seq.is_finished(None, sampling.max_new_tokens):
            t0 = time.perf_counter()
            key = torch.tensor([[seq.seq_id, acc, recovery]], dtype=torch.int32)
            self.draft_worker.submit(DraftRequest(DraftCommand.SERVE, key, torch.tensor([seq.num_tokens]),
                                                  torch.zeros((1, 1), dtype=torch.int32), torch.zeros(1),
                                                  prefix_tokens=[list(seq.token_ids)]))
            resp = self.draft_worker.get_response()
            spec = [int(t) for t in resp.spec_tokens[0].tolist()]
            spec_kp1 = torch.tensor([[recovery] + spec], dtype=torch.int32, device=self.target.dev)
            vres = self.target.verify(spec_kp1)
            vout = verify_greedy(vres.logits, spec_kp1)
            acc = int(vout.accept_until[0])
            recovery = int(vout.recovery_tokens[0])
            self.target.commit_tokens(spec[:acc] + [recovery])
            self._emit(seq, spec[:acc] + [recovery], sampling.max_new_tokens, on_token)
            collector.record_step(StepMetrics(target_verify_ms=(time.perf_counter() - t0) * 1000,
                                              cache_hit=bool(resp.cache_hit[0]), accepted_tokens=acc + 1))
        return seq.completion_token_ids
