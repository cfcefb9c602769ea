"""Tensor parallelism across GPUs: 2 ranks (and 4 / 8 when the machine has them).

Runs ``tests/tp_worker.py`` under torch.distributed.run; each rank compares its
sharded forward with the unsharded forward of the same weights on its GPU
(bf16 tolerance), all ranks must hold bit-identical logits, greedy SD on the
sharded pair must reproduce sharded AR, and the fused all-reduce must equal the
rank-order sum of the ranks' partials bit for bit (5, 40 and 224 rows).
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_ranks(world, tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           str(HERE / "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TP_RESULT_DIR=str(tmp_path))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = [json.loads((tmp_path / f"rank{i}.json").read_text()) for i in range(world)]
    print(json.dumps([{k: v for k, v in o.items() if k != "ar"} for o in res]))
    assert len(res) == world
    for o in res:
        assert o["status"] == 0
        for name in ("tp-target", "tp-draft"):
            e = o[name]
            assert e["ranks_identical"], (o["rank"], name)
            assert e["max_diff"] <= 2e-2 * max(e["scale"], 1.0), (o["rank"], name, e)
        assert o["sd_equals_ar"] and o["self_sd_equals_ar"], o
        assert all(o["allreduce_exact"].values()), (o["rank"], o["allreduce_exact"])
        assert o["ar"] == res[0]["ar"]
        assert o["self_sd_steps"] < 32
