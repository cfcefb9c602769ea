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
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", torch.cuda.current_device())
    import datetime

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from ssd_b200.kernels.kv_cache import KVCacheState
    from ssd_b200.models.gemma import PRESETS, GemmaRunner, GemmaWeights
    from ssd_b200.runtime.speculative import GreedyDecoder, SpeculativeDecoder
    from ssd_b200.runtime.tensor_parallel import TPComm, shard_weights

    comm = TPComm(heap_bytes=64 << 20, max_m=256, max_n=4096, device=dev)
    out = {"rank": rank}
    for name in ("tp-target", "tp-draft"):
        s = PRESETS[name]
        full = GemmaWeights.random(s, seed=31, device=dev, max_pos=512)
        local = shard_weights(full, rank, world)
        toks = torch.arange(3, 3 + 29, device=dev, dtype=torch.int32)[None] % s.vocab
        res = {}
        for tag, w, c in (("full", full, None), ("tp", local, comm)):
            ls = w.shape
            cache = KVCacheState.allocate(ls.num_layers, 8, 16, ls.num_kv_heads, ls.head_dim, torch.bfloat16, dev)
            table = torch.arange(8, dtype=torch.int32, device=dev)[None]
            lg = comm.alloc((1, 29, s.vocab)) if c is not None else torch.empty((1, 29, s.vocab), device=dev)
            GemmaRunner(w, 1, 64, 128, comm=c).forward(toks, torch.zeros(1, dtype=torch.int32, device=dev),
                                                       cache.pages, table, lg)
            torch.cuda.synchronize()
            res[tag] = lg.float().cpu()
        diff = (res["tp"] - res["full"]).abs().max().item()
        scale = res["full"].abs().max().item()
        gathered = [torch.empty_like(res["tp"]) for _ in range(world)]
        dist.all_gather(gathered, res["tp"])
        same = all(torch.equal(g, gathered[0]) for g in gathered)
        out[name] = {"max_diff": diff, "scale": scale, "ranks_identical": same}
    # SD == AR on the sharded pair (graph replay included)
    t = shard_weights(GemmaWeights.random(PRESETS["tp-target"], seed=41, device=dev, max_pos=512), rank, world)
    d = shard_weights(GemmaWeights.random(PRESETS["tp-draft"], seed=42, device=dev, max_pos=512), rank, world)
    prompt = list(range(50, 90))
    ar = GreedyDecoder(t, max_seq_len=256, comm=comm).generate(prompt, 32)
    sd, _ = SpeculativeDecoder(t, d, k=4, max_seq_len=256, comm=comm).generate(prompt, 32)
    self_sd, st = SpeculativeDecoder(t, t, k=4, max_seq_len=256, comm=comm).generate(prompt, 32)
    out["ar"] = ar
    out["sd_equals_ar"] = sd == ar
    out["self_sd_equals_ar"] = self_sd == ar
    out["self_sd_steps"] = st["steps"]
    torch.cuda.synchronize()
    out["status"] = comm.status()
    Path(os.environ["TP_RESULT_DIR"], f"rank{rank}.json").write_text(json.dumps(out))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
