"""Tensor-parallel host logic on CPU: weight sharding + the sharded forward, 2 gloo ranks.

Each rank shards the folded weights with ``runtime.tensor_parallel.shard_weights``
(the code the GPU path ships), runs the oracle's tensor-parallel restatement
(O/down partials summed with a gloo all-reduce, LM-head column blocks
all-gathered) and compares the logits with the unsharded oracle.  Covers both
head layouts: KV heads split across ranks (multi-head) and one replicated KV
head (multi-query).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gemma as og
from ssd_b200.models.gemma import PRESETS, GemmaWeights
from ssd_b200.runtime.tensor_parallel import shard_layout, shard_weights


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oshape(s):
    return og.GemmaShape(s.num_layers, s.d_model, s.num_heads, s.num_kv_heads, s.head_dim, s.ffn, s.vocab, s.eps,
                         s.rope_theta)


def _run(rank, world, port, preset, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape = PRESETS[preset]
        host = og.fold_norms(og.init_weights(_oshape(shape), seed=5))
        full = GemmaWeights.from_canonical(shape, host, dtype=torch.float32, device="cpu", max_pos=512)
        local = shard_weights(full, rank, world)
        lshape, blk = shard_layout(shape, rank, world)
        assert local.shape == lshape and (local.tp_rank, local.tp_world) == (rank, world)

        def allreduce(y):
            t = torch.from_numpy(np.ascontiguousarray(y))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(y):
            parts = [torch.empty_like(torch.from_numpy(y)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y)))
            return np.concatenate([p.numpy() for p in parts], axis=-1)

        rng = np.random.default_rng(3)
        toks = rng.integers(0, shape.vocab, size=(2, 7))
        table = np.arange(8, dtype=np.int32)[None, :].repeat(2, 0)
        table[1] = np.arange(8, 16)
        ref = og.OracleGemma(_oshape(shape), host, "fp32", max_pos=512)
        want = ref.forward(toks, og.new_pages(_oshape(shape), 16, 16), table, [0, 0])
        tp = og.OracleGemma(_oshape(lshape), local.to_canonical(), "fp32", max_pos=512)
        got = tp.forward(toks, og.new_pages(_oshape(lshape), 16, 16), table, [0, 0], allreduce=allreduce,
                         allgather=allgather, vocab_block=blk["vocab"])
        out_q.put((rank, float(np.abs(got - want).max()), float(np.abs(want).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("preset", ["tp-target", "tp-draft"])
def test_sharded_forward_matches_unsharded_oracle(preset):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, preset, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-4 * max(scale, 1.0), (rank, err, scale)


def test_shard_layout_blocks():
    s = PRESETS["gemma-7b"]
    loc, blk = shard_layout(s, 3, 8)
    assert (loc.num_heads, loc.num_kv_heads, loc.ffn, loc.vocab) == (2, 2, 3072, 256000)
    assert blk == {"q": (6, 2), "kv": (6, 2), "ffn": (9216, 3072), "vocab": (96000, 32000)}
    loc2, blk2 = shard_layout(PRESETS["gemma-2b"], 7, 8)
    assert (loc2.num_heads, loc2.num_kv_heads) == (1, 1) and blk2["kv"] == (0, 1)  # MQA: KV head replicated
    with pytest.raises(ValueError):
        shard_layout(PRESETS["gemma-7b"], 0, 3)
