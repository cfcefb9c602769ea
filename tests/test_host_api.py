"""Host-side API pieces that need no GPU: config, sampling params, branch prior, metrics."""

from __future__ import annotations

import torch

from ssd_b200.algorithm.branch_prior import build_branch_keys, expand_fanout_branches, top_f_recovery_tokens
from ssd_b200.config import DecodeMode, SSDConfig
from ssd_b200.runtime.metrics import MetricsCollector, StepMetrics
from ssd_b200.sampling_params import SamplingParams


def test_config_mq_len_and_fanout_string():
    assert SSDConfig().mq_len == 10  # (2,2,2,2,2), k=4
    c = SSDConfig.from_fanout_string("3,3,3,3,3", mode=DecodeMode.SSD)
    assert c.fan_out_list == (3, 3, 3, 3, 3) and c.mq_len == 15
    assert SSDConfig(speculate_k=6, fan_out_list=(2, 1)).mq_len == 2 + 6 * 1
    assert DecodeMode("ssd") is DecodeMode.SSD


def test_sampling_params_defaults():
    s = SamplingParams()
    assert s.max_new_tokens > 0 and s.temperature >= 0


def test_branch_prior_topf_and_expand():
    lg = torch.tensor([[0.1, 3.0, -1.0, 2.0], [5.0, 0.0, 4.0, 1.0]])
    top = top_f_recovery_tokens(lg, 2)
    assert top.tolist() == [[1, 3], [0, 2]] and top.dtype == torch.int32
    assert top_f_recovery_tokens(lg[:, None, :].expand(2, 3, 4), 1).tolist() == [[1], [0]]
    base = build_branch_keys(torch.tensor([7, 8]), torch.tensor([0, 0]), torch.tensor([1, 1]))
    keys, mq = expand_fanout_branches(base, (2, 1), top)
    assert mq == 3
    assert keys.tolist() == [[7, 0, 1], [8, 0, 0], [7, 0, 3], [8, 0, 2], [7, 1, 1], [8, 1, 0]]


def test_metrics_collector():
    m = MetricsCollector("sd")
    m.start()
    m.record_first_token()
    m.record_step(StepMetrics(accepted_tokens=3, cache_hit=True, verify_device_ms=2.0))
    m.record_step(StepMetrics(accepted_tokens=1))
    m.record_accepts([2, 0])
    live = m.metrics
    assert live.total_tokens == 4 and live.total_time_s >= 0.0
    r = m.finish()
    assert r.total_tokens == 4 and r.accepted_per_step == 2.0 and r.cache_hit_rate == 0.5
    assert r.ttft_s <= r.total_time_s and r.verify_device_ms == 2.0
    d = r.to_dict()
    assert d["num_steps"] == 2 and d["accept_histogram"] == {0: 1, 2: 1}
    # a batched step advances several sequences: accepted_per_step is per sequence-step
    m2 = MetricsCollector("sd")
    m2.start()
    m2.record_step(StepMetrics(accepted_tokens=8, sequences=4))
    assert m2.finish().accepted_per_step == 2.0


def test_slot_scheduler_refills_freed_slots():
    from ssd_b200.runtime.scheduler import Scheduler
    from ssd_b200.runtime.sequence import SequenceStatus

    s = Scheduler(num_slots=2)
    seqs = [s.add_request([i, i + 1]) for i in range(5)]
    assert [q.seq_id for q in seqs] == list(range(5)) and s.has_work()
    placed = s.admit()
    assert [(i, q.seq_id) for i, q in placed] == [(0, 0), (1, 1)] and s.admit() == []
    assert all(q.status is SequenceStatus.RUNNING for _, q in placed)
    assert s.retire(1).seq_id == 1 and seqs[1].status is SequenceStatus.FINISHED
    assert [(i, q.seq_id) for i, q in s.admit()] == [(1, 2)]
    s.retire(0)
    s.retire(1)
    assert [(i, q.seq_id) for i, q in s.admit()] == [(0, 3), (1, 4)]
    s.retire(0)
    assert s.slots() == [(1, seqs[4])] and s.free_slots() == [0] and s.has_work()
    s.retire(1)
    assert not s.has_work() and [q.seq_id for q in s.finished] == [1, 0, 2, 3, 4]


def test_draft_worker_yields_only_to_requests_it_cannot_serve():
    """The cache rebuild keeps going while the queued request's keys are all being drafted,
    and stops for a request (or a shutdown) it cannot serve."""
    from ssd_b200.algorithm.async_protocol import DraftCommand, DraftRequest
    from ssd_b200.runtime.workers import DraftWorker

    w = DraftWorker(SSDConfig(), draft_model=None)
    drafting = {(7, 0, 11), (7, 1, 12), (7, 4, 3)}
    assert not w._next_request_misses(drafting)  # nothing queued

    def req(keys, cmd=DraftCommand.SERVE):
        z = torch.zeros(0)
        return DraftRequest(cmd, torch.tensor(keys, dtype=torch.int32), z, z, z)

    w.submit(req([[7, 1, 12]]))
    assert not w._next_request_misses(drafting)  # its key is being drafted: finish and hit
    assert w._next_request_misses(set())
    w.request_queue.get()
    w.submit(req([[7, 1, 13]]))
    assert w._next_request_misses(drafting)  # a miss either way: yield to it now
    w.request_queue.get()
    w.submit(req([[7, 0, 11], [7, 2, 5]]))
    assert w._next_request_misses(drafting)  # one row of the request is not covered
    w.request_queue.get()
    w.submit(req(torch.zeros((0, 3)).tolist(), DraftCommand.SHUTDOWN))
    assert w._next_request_misses(drafting)
