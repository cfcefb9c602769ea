"""Draft worker with host queues for async SSD (jax_ssd/runtime/workers.py:32-145).

The worker thread serves ``DraftRequest(SERVE)`` messages on its own CUDA
stream:

1. ``_handle`` looks the request keys ``[seq_id, accepted, recovery]`` up in its
   ``SpecCache`` (``ssd_spec_cache_lookup``); on a miss it drafts k tokens from
   the request's committed prefix (``draft_speculate``) -- the reference drafts
   from ``[recovery]`` alone (workers.py:96-109).
2. After the response is queued, ``_rebuild_cache`` resets the cache and
   pre-drafts the branches the next request can name while the target
   verifies: for each accepted length ``a`` in 0..k, ``fan_out_list[a]``
   recovery candidates, the top tokens of the draft's own distribution at
   position ``a`` with the drafted token removed (a rejected draft is never the
   recovery token; at ``a = k`` the bonus distribution is used as is).  Each
   branch is drafted from ``prefix + spec[:a] + [candidate]``, so a hit serves
   exactly the tokens a miss would draft.  All branches of a request are
   drafted together (``GemmaAdapter.draft_branches``: the committed prefix is
   forked into branch rows that share its KV pages, then k batched forwards --
   the paged attention over forked tables is the reference's branch mask,
   jax_ssd/kernels/masks.py:8-30).  The rebuild overlaps the target's verify when
   the engine runs the draft on another device or stream.  It yields to the next
   request as soon as that request names a key the rebuild is not drafting (the
   rebuild cannot serve it, so finishing would only delay its miss draft); a
   request whose key is being drafted waits for the rebuild and hits.  Results do
   not depend on this: a hit serves the tokens a miss would draft.  A miss drafts
   k tokens and responds; the bonus forward the rebuild needs for the a = k
   candidates runs after the response, off the request's path.  The reference
   (which rebuilds inside ``_handle``) builds the same keys
   (workers.py:119-145) from top-F of all-zero glue logits, i.e. candidates
   ``0..F-1``, and drafts them from the candidate alone.
"""

from __future__ import annotations

import queue
import threading
from dataclasses import dataclass

import torch

from ..algorithm.async_protocol import DraftCommand, DraftRequest, DraftResponse
from ..algorithm.spec_cache import SpecCache
from ..config import SSDConfig


@dataclass
class WorkerConfig:
    """Worker options of the reference (workers.py:26-29); carried for callers that build one."""

    use_toy: bool = True
    instance_mode: bool = False


class DraftWorker:
    def __init__(self, config: SSDConfig, draft_model) -> None:
        self.config = config
        self.model = draft_model
        self.request_queue: queue.Queue = queue.Queue()
        self.response_queue: queue.Queue = queue.Queue()
        self.cache: SpecCache | None = None
        self.stream: torch.cuda.Stream | None = None
        self._thread: threading.Thread | None = None
        self._running = False
        self.error: BaseException | None = None
        self.prefetch = True
        self.branches_drafted = 0
        self._context_tokens: list[int] = []

    def set_context(self, tokens: list[int]) -> None:
        """Record the sequence's context tokens (workers.py:62-63).  Requests carry their own
        committed prefix here, so drafting does not read it."""
        self._context_tokens = [int(t) for t in tokens]

    def start(self) -> None:
        self._running = True
        dev = torch.device(self.model.dev)
        self._device = dev.index if dev.index is not None else torch.cuda.current_device()
        self.stream = torch.cuda.Stream(device=self._device)
        with torch.cuda.device(self._device), torch.cuda.stream(self.stream):
            self.cache = SpecCache.create(num_branches=max(1, self.config.mq_len), k=self.config.speculate_k,
                                          vocab=self.model.vocab_size, device=self.model.dev, with_logits=False)
        self.stream.synchronize()
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._running = False
        if self._thread:
            self.request_queue.put(DraftRequest(DraftCommand.SHUTDOWN, torch.zeros((0, 3), dtype=torch.int32),
                                                torch.zeros(0), torch.zeros(0), torch.zeros(0)))
            self._thread.join(timeout=30)

    def submit(self, req: DraftRequest) -> None:
        self.request_queue.put(req)

    def get_response(self, timeout: float = 120.0) -> DraftResponse:
        resp = self.response_queue.get(timeout=timeout)
        if isinstance(resp, BaseException):
            raise resp
        return resp

    def _loop(self) -> None:
        try:
            torch.cuda.set_device(self._device)
        except BaseException as exc:
            self.error = exc
            self.response_queue.put(exc)
            return
        with torch.cuda.stream(self.stream):
            while self._running:
                try:
                    req = self.request_queue.get(timeout=0.1)
                except queue.Empty:
                    continue
                if req.command == DraftCommand.SHUTDOWN:
                    break
                try:
                    resp, plans = self._handle(req)
                    self.response_queue.put(resp)
                    if self.prefetch:
                        self._rebuild_cache(plans)
                except BaseException as exc:  # surface to the engine thread
                    self.error = exc
                    self.response_queue.put(exc)

    def _handle(self, req: DraftRequest) -> tuple[DraftResponse, list]:
        k = self.config.speculate_k
        hit, _, tokens, _ = self.cache.lookup(req.cache_keys)
        hit_h = hit.cpu()
        keys_h = req.cache_keys.cpu()
        rows, plans = [], []
        for i in range(keys_h.shape[0]):
            prefix = [int(t) for t in req.prefix_tokens[i]]
            if bool(hit_h[i]):
                spec = [int(t) for t in tokens[i].tolist()]
                rows.append(tokens[i])
                plans.append((keys_h[i], prefix, spec, None))
                continue
            spec, logits = self.model.draft_speculate(prefix, k)
            rows.append(torch.tensor(spec, dtype=torch.int32, device=self.model.dev))
            plans.append((keys_h[i], prefix, spec, logits))  # logits [k, V]: the bonus row comes later
        spec_tokens = torch.stack(rows)
        self.stream.synchronize()
        return DraftResponse(cache_hit=hit, spec_tokens=spec_tokens,
                             draft_logits=torch.zeros((len(rows), k, 1), dtype=torch.float32)), plans

    def _next_request_misses(self, drafting: set) -> bool:
        """True when a request is queued and one of its keys is not in ``drafting``."""
        with self.request_queue.mutex:
            if not self.request_queue.queue:
                return False
            req = self.request_queue.queue[0]
        if req.command != DraftCommand.SERVE:
            return True
        keys = {tuple(int(v) for v in row) for row in req.cache_keys.reshape(-1, 3).tolist()}
        return not keys <= drafting

    def _rebuild_cache(self, plans: list) -> None:
        """Pre-draft the next request's branches (see the module docstring).

        Branches are drafted most-likely first, scored with the draft's own
        distribution q standing in for the target's: an accepted length ``a``
        has weight prod_{j<a} q_j(s_j) * (1 - q_a(s_a)) (prod_{j<k} q_j(s_j) for
        a = k) and candidate c at ``a`` the share q_a(c) / (1 - q_a(s_a)).
        """
        k = self.config.speculate_k
        fan = tuple(self.config.fan_out_list)
        if len(fan) < k + 1:
            fan = fan + (fan[-1],) * (k + 1 - len(fan))
        self.cache.reset()
        nothing: set = set()
        branches = []
        for key, prefix, spec, logits in plans:
            if self._next_request_misses(nothing):  # the cache is empty: nothing to wait for
                return
            if logits is None:  # served from the cache: draft once more for the glue logits
                spec, logits = self.model.draft_speculate(prefix, k, with_bonus=True)
            elif logits.shape[0] == k:  # a miss: the bonus row (one forward over the last draft)
                _, bonus = self.model.draft_speculate(prefix + spec, 0, with_bonus=True)
                logits = torch.cat([logits, bonus])
            q = torch.softmax(logits.float(), dim=-1)
            q_spec = q[torch.arange(k, device=q.device), torch.tensor(spec, device=q.device)].tolist()
            reach = 1.0  # prod_{j<a} q_j(s_j)
            for a in range(k + 1):
                row = q[a].clone()
                if a < k:
                    row[spec[a]] = 0.0  # a rejected draft is never the recovery token
                if fan[a] > 0:
                    top = torch.topk(row, fan[a])
                    for c, pc in zip(top.indices.tolist(), top.values.tolist()):
                        # reach * (1 - q_a(s_a)) * q_a(c) / (1 - q_a(s_a)) = reach * q_a(c)
                        branches.append((reach * pc, int(key[0]), a, int(c), spec[:a] + [int(c)], prefix))
                if a < k:
                    reach *= q_spec[a]
        branches.sort(key=lambda b: -b[0])
        chosen = branches[: self.cache.keys.shape[0]]
        drafting = {(sid, a, c) for _, sid, a, c, _f, _p in chosen}
        stop = lambda: self._next_request_misses(drafting)  # noqa: E731
        by_prefix: dict[int, list] = {}
        for slot, br in enumerate(chosen):
            by_prefix.setdefault(id(br[5]), []).append((slot, br))
        for group in by_prefix.values():
            prefix = group[0][1][5]
            if hasattr(self.model, "draft_branches"):
                # every branch of one request at once: forked trunk pages, batched draft forwards
                specs = self.model.draft_branches(prefix, [br[4] for _, br in group], k, stop=stop)
            else:
                specs = []
                for _, br in group:
                    if stop():
                        break
                    specs.append(self.model.draft_speculate(prefix + br[4], k)[0])
            for (slot, (_, sid, a, c, _feed, _p)), sp in zip(group, specs):
                self.cache.insert(slot, [sid, a, c], sp)
                self.branches_drafted += 1
            if len(specs) < len(group):  # yielded to a request the rebuild cannot serve
                break
        self.stream.synchronize()
