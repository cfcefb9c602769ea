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
    m.record_step(StepMetrics(accepted_tokens=3, cache_hit=True))
    m.record_step(StepMetrics(accepted_tokens=1))
    r = m.finish()
    assert r.total_tokens == 4 and r.accepted_per_step == 2.0 and r.cache_hit_rate == 0.5
    assert r.to_dict()["num_steps"] == 2
