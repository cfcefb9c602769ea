"""One rank of the multi-GPU tensor-parallel check (launched by test_gpu_tp_multi.py
through torch.distributed.run); writes rank<r>.json into $TP_RESULT_DIR."""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "ssd-tpu-_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> None:
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    import datetime

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from ssd_b200.runtime.tensor_parallel import tp_selfcheck

    def gather(t):
        parts = [torch.empty_like(t.cpu()) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, t.cpu())
        return parts

    out = tp_selfcheck(gather)
    out["rank"] = rank
    Path(os.environ["TP_RESULT_DIR"], f"rank{rank}.json").write_text(json.dumps(out))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
