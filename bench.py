#!/usr/bin/env python
"""Benchmark: greedy speculative decoding, random-init Gemma-7B target + Gemma-2B draft,
k = 4, batch 1, prompt of 128 random tokens (the 1-GPU sd workload of the verify path).

One bench step = one speculative iteration: k draft forwards of the 2B, one
verify forward of the 7B over k+1 tokens, fused greedy acceptance, page
rollback of both caches, and the 8-byte read of (accepted, recovery).

Prints ONE JSON line (rank 0).  ``value`` = committed tokens/s over the K timed
steps (all ranks, device-timed with CUDA events, max over ranks); ``e2e`` = the
same metric for a whole ``SpeculativeDecoder.generate`` call from a host prompt
list to host tokens (prefill included); ``verify_step_us`` / ``verify_hbm_gbs``
describe the verify forward alone; ``roofline`` covers the dominant kernel (the
weight-streaming projections).  With N > 1 (torchrun) the pair is tensor-parallel
over the N GPUs (``--parallel tp``, the default: heads / FFN / vocabulary split,
the O / down all-reduces and the LM-head all-gather fused into the projection
kernels over NVLink; one sequence, strong scaling), or each rank decodes its own
sequence (``--parallel replicas``; no data-path collective, weak scaling).

``--impl reference`` times the CPU restatement of the same path (numpy oracle:
the reference's own JAX code cannot run here) on a bounded layer sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ssd-tpu-_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "Gemma-7B/2B sd tokens/sec at TP 1/2/4/8 B200; verify-step µs; HBM GB/s"
WORKLOAD = "gemma-7b target + gemma-2b draft, random-init bf16, sd greedy k=4, batch 1, prompt 128"
PEAKS = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_RATIO = 309.07 / 302.52  # DRAM bytes / algorithmic bytes of one captured 7B gate/up launch


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--e2e-new-tokens", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", choices=["tp", "replicas"], default="tp",
                    help="N > 1: tensor-parallel pair (one sequence) or independent replicas")
    ap.add_argument("--op", choices=["linear", "attention", "verify", "sample", "topp", "allreduce", "allgather"],
                    default=None,
                    help="time one kernel family on its op-level workload instead of the decode loop")
    ap.add_argument("--rows", "--m", dest="m", type=int, default=5)
    ap.add_argument("--cols", "--n", dest="n", type=int, default=49152)
    ap.add_argument("--depth", "--kdim", dest="kdim", type=int, default=3072)
    ap.add_argument("--batch", type=int, default=0,
                    help="> 0: batched serving workload (B sequences, --k drafts, --temperature, contexts "
                         "U[--ctx-min, --ctx-max]); prints its own JSON line instead of the decode-loop line")
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-p", dest="top_p", type=float, default=0.95,
                    help="batched mode: top-p nucleus of the draft and target distributions (1 = off)")
    ap.add_argument("--ctx-min", type=int, default=1024)
    ap.add_argument("--ctx-max", type=int, default=8192)
    ap.add_argument("--attn", choices=["2a", "decode7b", "decode2b"], default="2a",
                    help="--op attention shape: op config 2a (B=8, ctx U[512,4096]) or one decode step")
    return ap.parse_args()


def peaks():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU leg
def cpu_sample_rate(k: int, tokens_per_step: float, target_w=None, draft_w=None, prompt_len: int = 128):
    """Time the numpy oracle on a layer sample of the workload and scale to full depth.

    Sample: 2 of the 28 Gemma-7B layers + its LM head (verify over k+1 tokens)
    and 1 of the 18 Gemma-2B layers + its LM head (one draft decode), both
    after a prompt of ``prompt_len`` tokens, fp32 numpy with all host threads.
    Returns (tokens/s, step seconds, description).
    """
    import numpy as np

    from oracle.gemma import GemmaShape as OShape
    from oracle.gemma import OracleGemma, init_weights, new_pages

    full_t, full_d = 28, 18
    st = OShape(2, 3072, 16, 16, 256, 24576, 256000)
    sd = OShape(1, 2048, 8, 1, 256, 16384, 256000)
    wt = target_w if target_w is not None else init_weights(st, 1)
    wd = draft_w if draft_w is not None else init_weights(sd, 2)
    mt, md = OracleGemma(st, wt, "fp32"), OracleGemma(sd, wd, "fp32")
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 256000, prompt_len)[None]
    nb = (prompt_len + 64) // 16 + 2
    table = np.arange(nb, dtype=np.int32)[None]
    pt, pd = new_pages(st, nb, 16), new_pages(sd, nb, 16)
    mt.forward(prompt, pt, table, [0], with_head=False)
    md.forward(prompt, pd, table, [0], with_head=False)
    tv, td = {}, {}
    mt.forward(rng.integers(0, 256000, (1, k + 1)), pt, table, [prompt_len], timings=tv)
    md.forward(rng.integers(0, 256000, (1, 1)), pd, table, [prompt_len], timings=td)
    verify_s = tv["layers_s"] * full_t / st.num_layers + tv["head_s"]
    draft_s = td["layers_s"] * full_d / sd.num_layers + td["head_s"]
    step_s = k * draft_s + verify_s
    desc = (f"numpy oracle, fp32: 2/28 Gemma-7B layers + LM head (verify, {k + 1} tokens) and 1/18 Gemma-2B "
            f"layers + LM head (draft decode) after a {prompt_len}-token prompt, layer time scaled to full "
            f"depth; step = {k} draft decodes + 1 verify; {tokens_per_step:.2f} tokens/step")
    return tokens_per_step / step_s, step_s, desc


def run_reference(args):
    """--impl reference: the CPU restatement of the path, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle.gemma import GemmaShape as OShape
    from oracle.gemma import init_weights

    wt = init_weights(OShape(2, 3072, 16, 16, 256, 24576, 256000), 1)
    wd = init_weights(OShape(1, 2048, 8, 1, 256, 16384, 256000), 2)
    rates, steps = [], []
    t0 = time.perf_counter()
    n = 0
    for i in range(args.warmup + args.steps):
        rate, step_s, desc = cpu_sample_rate(args.k, 1.0, wt, wd, args.prompt_len)
        if i >= args.warmup:
            rates.append(rate)
            steps.append(step_s)
            n += 1
        if time.perf_counter() - t0 > 90 and n >= 1:
            break
    value = float(np.mean(rates))
    cores = os.cpu_count()
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "ms_per_step": 1000.0 * float(np.mean(steps)), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": args.prompt_len,
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": desc + f"; {n} timed samples (1 accepted+recovery token per step assumed)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU leg
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from ssd_b200.models.gemma import PRESETS, GemmaRunner, GemmaWeights, ProjectionTimer
    from ssd_b200.runtime.speculative import SpeculativeDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    k = args.k
    tp = world > 1 and args.parallel == "tp"
    st_, sd_ = PRESETS["gemma-7b"], PRESETS["gemma-2b"]
    comm = None
    if tp:
        from ssd_b200.runtime.tensor_parallel import TPComm, shard_weights

        # every rank draws the same full weights from the seed and keeps its shard
        target = shard_weights(GemmaWeights.random(st_, seed=1000), rank, world)
        draft = shard_weights(GemmaWeights.random(sd_, seed=2000), rank, world)
        torch.cuda.empty_cache()
        comm = TPComm(heap_bytes=192 << 20, max_m=64, max_n=max(st_.d_model, sd_.d_model))
        rng = np.random.default_rng(0)
    else:
        target = GemmaWeights.random(st_, seed=1000 + rank)
        draft = GemmaWeights.random(sd_, seed=2000 + rank)
        rng = np.random.default_rng(rank)
    lt, ld = target.shape, draft.shape  # this rank's (sharded) shapes
    prompt = [int(x) for x in rng.integers(0, st_.vocab, args.prompt_len)]
    total_steps = args.warmup + args.steps
    max_seq = args.prompt_len + (total_steps + 2) * (k + 1) + 32
    max_seq = max(max_seq, args.prompt_len + args.e2e_new_tokens * (k + 1) + 32)
    dec = SpeculativeDecoder(target, draft, k=k, max_seq_len=max_seq, comm=comm)
    dec.start(prompt)
    for _ in range(args.warmup):
        dec.step()
    stream = torch.cuda.current_stream()
    verify_ms = []
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    torch.cuda.nvtx.range_push("timed")
    tokens = 0
    accepted = 0
    ctx_sum = 0
    for i in range(args.steps):
        ctx_sum += dec.t.n + k + 1
        new = dec.step()
        verify_ms.append(dec.last_verify_ms)
        tokens += len(new)
        accepted += dec.last_accept
    torch.cuda.nvtx.range_pop()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    # max time / total tokens over ranks
    t = torch.tensor([ms, float(tokens)], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = t[0:1].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t[1:2].clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        ms_max, tok_all = float(tmax.item()), float(tsum.item())
        if tp:
            tok_all = float(tokens)  # one sequence decoded by all ranks together
    else:
        ms_max, tok_all = ms, float(tokens)
    value = tok_all / (ms_max / 1000.0)

    # Projection launches timed with CUDA events in a second window of the same
    # decode (events between kernels add gaps, so they stay out of `value`).
    timer = ProjectionTimer(capacity=4 * st_.num_layers + 8)
    if comm is not None:
        heap_top = comm._top
    dec_p = SpeculativeDecoder(target, draft, k=k, max_seq_len=max_seq, timer=timer, comm=comm)
    dec_p.start(prompt)
    for _ in range(args.warmup):
        dec_p.step()
    timer.reset()
    for _ in range(max(8, min(args.steps, 32))):
        dec_p.step()
    torch.cuda.synchronize()
    del dec_p
    if comm is not None:
        comm._top = heap_top  # the profiled decoder's symmetric buffers are free again

    # verify-step bytes (per rank): its target weight shard once + its KV rows read
    # (+ the logits block it writes); the replicated embedding is read for k+1 rows only
    wbytes = lt.layer_weight_bytes() * lt.num_layers + (st_.vocab // max(world if tp else 1, 1)) * st_.d_model * 2
    kv_tok = lt.kv_bytes_per_token()
    mean_ctx = ctx_sum / args.steps
    verify_bytes = wbytes + kv_tok * mean_ctx + (k + 1) * st_.vocab * 4
    verify_us = 1000.0 * statistics.mean(verify_ms)
    hbm_peak, peak_kind = peaks()

    # dominant kernel: the weight-streaming projections inside the timed verify forwards
    M = k + 1
    d, hq, hkv, D, F = lt.d_model, lt.num_heads, lt.num_kv_heads, lt.head_dim, lt.ffn
    V = st_.vocab // (world if tp else 1)
    shapes = {"qkv": ((hq + 2 * hkv) * D, d, 2), "o": (d, hq * D, 2), "gate_up": (2 * F, d, 2),
              "down": (d, F, 2), "lm_head": (V, d, 4)}
    proj_bytes = 0.0
    proj_ms = 0.0
    per_kind = {}
    for kind, (n_, k_, ob) in shapes.items():
        nl = timer.launches[kind]
        if nl == 0:
            continue
        out_cols = n_ // 2 if kind == "gate_up" else n_
        b1 = n_ * k_ * 2 + M * k_ * 2 + M * out_cols * ob + (M * n_ * 2 if kind in ("o", "down") else 0)
        proj_bytes += b1 * nl
        proj_ms += timer.total_ms[kind]
        per_kind[kind] = {"launches": nl, "us_per_launch": 1000.0 * timer.total_ms[kind] / nl,
                          "gbs": b1 * nl / (timer.total_ms[kind] / 1000.0) / 1e9}
    n_launch = sum(timer.launches.values())
    achieved = proj_bytes / (proj_ms / 1000.0) / 1e9
    lpf_t = GemmaRunner.launches_per_forward(lt, True, False)
    lpf_d = GemmaRunner.launches_per_forward(ld, True, True)
    launches_per_step = k * (lpf_d + 1) + 1 + (1 + lpf_t + 1) + 2

    # e2e: one whole generate() from a host prompt list to host tokens
    dec2 = SpeculativeDecoder(target, draft, k=k, max_seq_len=max_seq, comm=comm)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    out, info = dec2.generate(prompt, args.e2e_new_tokens)
    torch.cuda.synchronize()
    w1 = time.perf_counter()
    e2e_local = torch.tensor([w1 - w0, float(len(out))], dtype=torch.float64, device=dev)
    if world > 1:
        a = e2e_local[0:1].clone()
        dist.all_reduce(a, op=dist.ReduceOp.MAX)
        b = e2e_local[1:2].clone()
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
        e2e_val = (len(out) if tp else float(b.item())) / float(a.item())
    else:
        e2e_val = len(out) / (w1 - w0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            wt = target.to_canonical(layers=2)
            wd = draft.to_canonical(layers=1)
            rate, step_s, desc = cpu_sample_rate(k, tokens / args.steps, wt, wd, args.prompt_len)
            cpu = {"value": rate, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port", "sample": desc}
        except Exception as exc:  # the CPU leg is a reported baseline only
            cpu = {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {exc!r}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": {"workload": WORKLOAD, "global_batch": 1 if tp else world, "seq_len": args.prompt_len, "k": k,
                       "parallelism": f"tp{world}" if tp else ("replicas" if world > 1 else "tp1"),
                       "l2": "inputs larger than L2: 17.1 GB of target weights + 5.0 GB of draft weights "
                             "streamed per step"},
            "verify_step_us": verify_us,
            "verify_hbm_gbs": verify_bytes / (verify_us / 1e6) / 1e9,
            "verify_roofline_frac": (verify_bytes / (verify_us / 1e6) / 1e9) / hbm_peak,
            "accept_rate": accepted / (args.steps * k),
            "tokens_per_step": tokens / args.steps,
            "roofline": {"bound": "hbm", "kernel": "skinny projections (QKV, O, gate/up, down, LM head), "
                         f"M = {M}", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                         # DRAM bytes per launch: the gate/up ncu capture's read + write over its
                         # algorithmic bytes (309.07 / 302.52 MB), applied to the average launch
                         "traffic": TRAFFIC_RATIO * proj_bytes / max(n_launch, 1) if not tp else None,
                         "traffic_source": "ncu capture of the 7B gate/up launch (profiles/linear_tc_gate_up_m5.md): "
                                           "309.07 MB DRAM per 302.52 MB algorithmic, scaled to the average launch",
                         "window": "event-timed projection launches of a separate profiled decode window",
                         "per_launch_bytes": proj_bytes / max(n_launch, 1), "per_kind": per_kind},
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": 16 * 4 + 8 * 4,
                    "d2h_bytes_per_step": 2 * 4 + (k + 1) * 4, "new_tokens": len(out),
                    "api": "SpeculativeDecoder.generate(prompt list) -> token list"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        torch.cuda.synchronize()
        if comm.status() != 0:
            print(f"rank {rank}: tensor-parallel wait timed out", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


# ----------------------------------------------------------------- op-level legs
def run_op(args):
    """Op-level workloads (one JSON line each): the projection streamer on one shape, the
    paged verify attention (B=8, ctx U[512,4096], 16x256 heads, 5 queries) and the acceptance
    kernels (B=8, K=4, V=256000, logits ~ N(0, 3^2)).  Inputs exceed L2 or are rotated so
    every timed launch reads from HBM."""
    import numpy as np
    import torch

    from ssd_b200.algorithm.verify import verify_greedy, verify_sample
    from ssd_b200.kernels.kv_cache import KVCacheState, paged_verify_attention
    from ssd_b200.kernels.ops import linear

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    hbm, kind = peaks()
    g = torch.Generator(device="cuda").manual_seed(0)
    reps = max(args.steps, 1)
    st = torch.cuda.current_stream()

    def timed(fn, nrot):
        """Device time per call: nrot calls captured in one CUDA graph, replayed (no host gaps)."""
        for i in range(max(args.warmup, nrot)):
            fn(i % nrot)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(nrot):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(reps):
            graph.replay()
        b_.record(st)
        torch.cuda.synchronize()
        return a.elapsed_time(b_) / (reps * nrot)

    if args.op == "linear":
        m, n, k = args.m, args.n, args.kdim
        nrot = max(1, int(np.ceil(512e6 / (n * k * 2))))  # rotate weights over > 4x L2
        ws = [(torch.randn((n, k), device="cuda", generator=g) * 0.02).bfloat16() for _ in range(nrot)]
        x = torch.randn((m, k), device="cuda", generator=g).bfloat16()
        y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        ms = timed(lambda i: linear(x, ws[i], "store", out=y), nrot)
        nbytes = n * k * 2 + m * k * 2 + m * n * 2
        line = {"op": "linear", "m": m, "n": n, "k": k, "us": ms * 1000, "gbs": nbytes / ms / 1e6,
                "frac": nbytes / ms / 1e6 / hbm, "peak_kind": kind, "weights_rotated": nrot}
    elif args.op in ("allreduce", "allgather"):
        # one tensor-parallel projection per rank (M x N outputs, this rank's K / N block),
        # against the plain projection of the same local shape; --n / --kdim are the
        # LOCAL sizes (7B O at TP2: --n 3072 --kdim 2048; LM head at TP2: --op allgather
        # --n 128000 --kdim 3072)
        from ssd_b200.kernels.ops import linear_allgather, linear_allreduce
        from ssd_b200.runtime.tensor_parallel import TPComm

        m, n, k = args.m, args.n, args.kdim
        comm = TPComm(heap_bytes=(64 << 20) + 8 * m * n * world * 4, max_m=m, max_n=n if args.op == "allreduce" else 1)
        nrot = max(1, int(np.ceil(512e6 / (n * k * 2))))
        ws = [(torch.randn((n, k), device="cuda", generator=g) * 0.02).bfloat16() for _ in range(nrot)]
        x = torch.randn((m, k), device="cuda", generator=g).bfloat16()
        if args.op == "allreduce":
            y = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
            ms_plain = timed(lambda i: linear(x, ws[i], "residual", out=y), nrot)
            ms = timed(lambda i: linear_allreduce(x, ws[i], y, comm), nrot)
            nbytes = n * k * 2 + m * k * 2 + 2 * m * n * 2
        else:
            y = comm.alloc((m, n * world), torch.float32)
            yl = torch.empty((m, n), dtype=torch.float32, device="cuda")
            ms_plain = timed(lambda i: linear(x, ws[i], "store_f32", out=yl), nrot)
            ms = timed(lambda i: linear_allgather(x, ws[i], y, comm), nrot)
            nbytes = n * k * 2 + m * k * 2 + m * n * 4
        torch.cuda.synchronize()
        t = torch.tensor([ms, ms_plain], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_plain = float(t[0]), float(t[1])
        line = {"op": args.op, "world": world, "m": m, "n_local": n, "k_local": k, "us": ms * 1000,
                "us_plain": ms_plain * 1000, "collective_us": (ms - ms_plain) * 1000,
                "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm, "peak_kind": kind,
                "status": comm.status(), "weights_rotated": nrot}
        if world > 1:
            dist.barrier()
        comm.close()
        if rank != 0:
            return
    elif args.op == "attention":
        b, t, hq, hkv, d, bs = 8, 5, 16, 16, 256, 16
        rng = np.random.default_rng(0)
        ctx = rng.integers(512, 4097, b)
        if args.attn == "decode7b":
            b, ctx = 1, np.array([260])
        elif args.attn == "decode2b":
            b, t, hq, hkv, ctx = 1, 1, 8, 1, np.array([260])
        mb = int((ctx.max() + bs - 1) // bs)
        nb = b * mb
        cache = KVCacheState.allocate(1, nb, bs, hkv, d)
        cache.pages.normal_(generator=g)
        perm = torch.randperm(nb, generator=torch.Generator().manual_seed(0)).int().view(b, mb).cuda()
        q = torch.randn((b, t, hq, d), device="cuda", generator=g).bfloat16()
        sl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
        out = torch.empty_like(q)
        ms = timed(lambda i: paged_verify_attention(q, cache, 0, perm, sl, max_seq_len=mb * bs, out=out), 1)
        nbytes = int(ctx.sum()) * hkv * d * 2 * 2 + 2 * q.numel() * 2
        line = {"op": "paged_attention", "shape": args.attn, "B": b, "T": t, "Hq": hq, "Hkv": hkv, "ctx": ctx.tolist(), "us": ms * 1000, "gbs": nbytes / ms / 1e6,
                "frac": nbytes / ms / 1e6 / hbm, "peak_kind": kind, "kv_bytes": nbytes,
                "note": "KV pages (302 MB expected) exceed L2; one layer"}
    elif args.op in ("verify", "sample"):
        b, k, v = 8, 4, 256000
        nrot = 4
        lps = [3.0 * torch.randn((b, k + 1, v), device="cuda", generator=g) for _ in range(nrot)]
        spec = torch.randint(0, v, (b, k + 1), device="cuda", generator=g, dtype=torch.int32)
        if args.op == "verify":
            ms = timed(lambda i: verify_greedy(lps[i], spec), nrot)
            nbytes = b * (k + 1) * v * 4
        else:
            lqs = [3.0 * torch.randn((b, k, v), device="cuda", generator=g) for _ in range(nrot)]
            ua = torch.rand((b, k), device="cuda", generator=g)
            ug = torch.rand((b, v), device="cuda", generator=g).clamp_(1e-7, 1 - 1e-7)
            ms = timed(lambda i: verify_sample(lps[i], lqs[i], spec, (ua, ug)), nrot)
            nbytes = b * k * v * 4 + b * k * v * 4 + b * v * 4
        line = {"op": "verify_" + ("greedy" if args.op == "verify" else "sample"), "B": b, "K": k, "V": v,
                "us": ms * 1000, "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm, "peak_kind": kind,
                "algorithmic_bytes": nbytes}
    elif args.op == "topp":
        # top-p 0.95 at T = 1 over --rows rows of 256000 N(0, 3^2) logits; the mask works in place, so
        # every timed call gets a fresh copy (the copy is outside the events)
        from ssd_b200.algorithm.verify import top_p_mask_

        rows, v = args.m, 256000
        src = 3.0 * torch.randn((rows, v), device="cuda", generator=g)
        x = torch.empty_like(src)
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for i in range(args.warmup + reps):
            x.copy_(src)
            e0.record(st)
            top_p_mask_(x, 1.0, 0.95)
            e1.record(st)
            torch.cuda.synchronize()
            if i >= args.warmup:
                times.append(e0.elapsed_time(e1))
        ms = float(np.median(times))
        nbytes = rows * v * 4 * 2  # one read and one write of every logit
        line = {"op": "top_p_mask", "rows": rows, "V": v, "top_p": 0.95, "us": ms * 1000,
                "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm, "peak_kind": kind,
                "algorithmic_bytes": nbytes, "note": "rows copied fresh before each call (L2-warm when small)"}
    print(json.dumps(line), flush=True)


def run_batched(args):
    """Batched serving (B sequences, k drafts, sampling): Gemma-7B target + Gemma-2B draft, random-init
    bf16, contexts ~ U[ctx_min, ctx_max] stood in by seeded N(0, 1) K/V in both caches (a prefill of
    ~150 K tokens would take minutes and is not what the step measures).  One step = k draft forwards
    over B rows + one verify forward over B*(k+1) rows + rejection sampling + rollbacks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.runtime.batched import BatchedSpeculativeDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    B, k = args.batch, args.k
    st_, sd_ = PRESETS["gemma-7b"], PRESETS["gemma-2b"]
    comm = None
    if world > 1:
        from ssd_b200.runtime.tensor_parallel import TPComm, shard_weights

        target = shard_weights(GemmaWeights.random(st_, seed=1000, max_pos=args.ctx_max + 512), rank, world)
        draft = shard_weights(GemmaWeights.random(sd_, seed=2000, max_pos=args.ctx_max + 512), rank, world)
        torch.cuda.empty_cache()
        comm = TPComm(heap_bytes=1 << 30, max_m=max(256, B * (k + 1)), max_n=max(st_.d_model, sd_.d_model))
    else:
        target = GemmaWeights.random(st_, seed=1000, max_pos=args.ctx_max + 512)
        draft = GemmaWeights.random(sd_, seed=2000, max_pos=args.ctx_max + 512)
    rng = np.random.default_rng(0)
    ctx = [int(x) for x in rng.integers(args.ctx_min, args.ctx_max + 1, B)]
    steps = args.warmup + args.steps
    grow = (steps + 2) * (k + 1)
    max_seq = args.ctx_max + grow + 16
    blocks = sum((c + grow + 15) // 16 + 1 for c in ctx) + 2
    dec = BatchedSpeculativeDecoder(target, draft, batch=B, k=k, max_seq_len=max_seq,
                                    temperature=args.temperature, top_p=args.top_p, seed=7, comm=comm,
                                    num_blocks=blocks)
    dec.start_synthetic(ctx, np.random.default_rng(1))
    for _ in range(args.warmup):
        dec.step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    e0.record(stream)
    tokens = 0
    verify_ms = []
    ctx_sum = 0.0
    for _ in range(args.steps):
        ctx_sum += float(dec.t.n.sum())
        new = dec.step()
        tokens += sum(len(x) for x in new)
        verify_ms.append(dec.last_verify_ms)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    hbm, kind = peaks()
    lt, ld = target.shape, draft.shape
    mean_ctx = ctx_sum / args.steps / B
    w_t = lt.layer_weight_bytes() * lt.num_layers + (st_.vocab // world) * st_.d_model * 2
    w_d = ld.layer_weight_bytes() * ld.num_layers + (sd_.vocab // world) * sd_.d_model * 2
    kv_t = B * mean_ctx * lt.kv_bytes_per_token()
    kv_d = B * mean_ctx * ld.kv_bytes_per_token()
    step_bytes = w_t + kv_t + k * (w_d + kv_d)
    step_s = ms / 1000.0 / args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "batched sd tokens/s (Gemma-7B/2B, B sequences, k drafts, sampling)",
            "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "n/a", "dtype": "bf16",
            "data": "synthetic (random-init weights; contexts stood in by seeded N(0,1) K/V)",
            "config": {"workload": f"batched serving B={B}, k={k}, T={args.temperature}, ctx U[{args.ctx_min}, "
                                   f"{args.ctx_max}]", "parallelism": f"tp{world}",
                       "top_p": args.top_p if args.temperature > 0 and args.top_p < 1 else None},
            "tokens_per_step": tokens / args.steps, "accept_rate": None,
            "verify_ms": statistics.mean(verify_ms),
            "step_bytes_per_rank": step_bytes, "step_hbm_gbs": step_bytes / step_s / 1e9,
            "step_roofline_frac": step_bytes / step_s / 1e9 / hbm, "peak_kind": kind,
            "clocks": clk,
        }), flush=True)
    if world > 1:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.op is not None:
        run_op(args)
        return
    if args.batch > 0 and args.impl == "ours":
        run_batched(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
