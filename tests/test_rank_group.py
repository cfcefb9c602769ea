"""Host logic of the engine's rank group (one worker process per GPU) on CPU: commands reach every
rank in order, ranks can run gloo collectives among themselves, a rank that raises surfaces as an
error in the caller without breaking the group, and a rank that fails to start is reported.  The
per-rank state here is a stand-in class; the engine's ``RankState`` needs a GPU."""

from __future__ import annotations

import pytest

from ssd_b200.runtime.rank_group import RankGroup

FAKE = "test_rank_group:FakeState"


class FakeState:
    def __init__(self, cfg, rank, world, device):
        if cfg.get("fail_rank") == rank:
            raise ValueError("planted start failure")
        self.rank, self.world, self.device = rank, world, device
        self.acc = 0

    def add(self, x):
        self.acc += x * (self.rank + 1)
        return self.acc

    def all_reduce(self, x):
        import torch
        import torch.distributed as dist

        t = torch.tensor([float(x + self.rank)])
        dist.all_reduce(t)
        return float(t.item())

    def fail_on(self, r):
        if self.rank == r:
            raise ValueError("planted failure")
        return self.rank

    def close(self):
        pass


def test_commands_collectives_and_failures():
    g = RankGroup([3, 5], {}, state_cls=FAKE)
    try:
        assert g.world == 2
        assert g.call("add", 3) == [3, 6]
        assert g.call("all_reduce", 1) == [3.0, 3.0]
        with pytest.raises(RuntimeError, match="planted failure"):
            g.call("fail_on", 1)
        assert g.call("add", 1) == [4, 8]  # the group keeps serving after a rank raised
    finally:
        g.close()


def test_start_failure_is_reported():
    with pytest.raises(RuntimeError, match="planted start failure"):
        RankGroup([0, 1], {"fail_rank": 1}, state_cls=FAKE)
