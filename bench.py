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
the reference's own JAX code cannot run here), one full-depth step per step.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import sys
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
    ap.add_argument("--qk-pairs", action="store_true",
                    help="weights with rotation-paired q/k rows: RoPE + K/V write fused into the QKV projection")
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
    ap.add_argument("--mode", choices=["sd", "ssd"], default="sd",
                    help="ssd: the async ssd engine through LLM.generate in ONE process -- target "
                         "tensor-parallel over GPUs 0..--tp-1, draft and its worker on GPU --tp; prints "
                         "its own JSON line")
    ap.add_argument("--tp", type=int, default=2, help="--mode ssd: target tensor-parallel size")
    ap.add_argument("--fanout", type=int, default=3, help="--mode ssd: branches per accepted length")
    ap.add_argument("--new-tokens", type=int, default=512, help="--mode ssd: tokens generated")
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
    """SM clock, power and clock-event reasons of one GPU, polled through NVML every 25 ms by a
    background thread from ``start`` to ``stop`` (the timed region).  Reading them changes no
    setting.  Reports "NVML unavailable" when the binding is missing."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, cuda_index: int, period_s: float = 0.025, enabled: bool = True):
        # one sampler per node (rank 0): eight ranks each polling NVML every 10 ms slowed the
        # tensor-parallel step measurably (the run's end-to-end rate exceeded its timed rate)
        self.enabled = enabled
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples: list[tuple[float, float, int]] = []
        self.sm_max = None
        self._stop = None
        self._thread = None
        self._handle = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = getattr(torch.cuda.get_device_properties(self.cuda_index), "uuid", None)
        if uuid is not None:
            u = str(uuid)
            u = u if u.startswith("GPU-") else "GPU-" + u
            try:
                return pynvml.nvmlDeviceGetHandleByUUID(u)
            except Exception:
                pass
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = int(vis.split(",")[self.cuda_index]) if vis and vis.split(",")[0].isdigit() else self.cuda_index
        return pynvml.nvmlDeviceGetHandleByIndex(idx)

    def start(self):
        import threading

        if not self.enabled:
            return
        try:
            import pynvml

            self._handle = self._nvml_handle()
            h = self._handle
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self._handle = None
            return
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = int(get_reasons(h))
                    self.samples.append((sm, pw, rs))
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if not self.enabled:
            return {"sampled_by": "rank 0"}
        if self._handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=5)
        sm = [x[0] for x in self.samples]
        reasons = sorted({name for _, _, r in self.samples for name, bit in self.REASONS if r & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.sm_max,
                "power_w_max": max((x[1] for x in self.samples), default=None), "reasons": reasons,
                "samples": len(sm), "source": "NVML, 25 ms period, timed region only, rank 0's GPU"}


# ----------------------------------------------------------------- CPU leg
def cpu_threads() -> int:
    """Raise the BLAS / OpenMP pools to every core this process may run on (torch.distributed.run
    exports OMP_NUM_THREADS=1) and return the BLAS thread count actually in use."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        import numpy  # noqa: F401  (loads the BLAS whose pool is resized)

        threadpool_limits(limits=n)
        blas = [i["num_threads"] for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(blas) if blas else n
    except Exception:
        return n


class CpuPipeline:
    """The workload's speculative step on the numpy oracle, at full depth, on the host cores.

    Target Gemma-7B (28 layers) and draft Gemma-2B (18 layers), fp32, after a ``prompt_len``-token
    prompt; one step = k one-token draft forwards + one target forward over k+1 tokens (+ both LM
    heads), at the positions the decode has reached.  To keep host memory small, the layers of a
    model cycle through the weights of ``sample_layers`` distinct layers (the same shapes, so the
    same arithmetic and the same bytes streamed per layer); the KV pages hold all layers.
    """

    def __init__(self, k: int, prompt_len: int, target_w=None, draft_w=None, steps: int = 64):
        import numpy as np

        from oracle.gemma import GemmaShape as OShape
        from oracle.gemma import OracleGemma, init_weights, new_pages

        self.k = k
        st = OShape(28, 3072, 16, 16, 256, 24576, 256000)
        sd = OShape(18, 2048, 8, 1, 256, 16384, 256000)
        wt = target_w if target_w is not None else init_weights(dataclasses.replace(st, num_layers=2), 1)
        wd = draft_w if draft_w is not None else init_weights(dataclasses.replace(sd, num_layers=1), 2)
        self.sample_layers = (len(wt["layers"]), len(wd["layers"]))
        lt, ld = wt["layers"], wd["layers"]
        wt = {**wt, "layers": lambda i: lt[i % len(lt)]}
        wd = {**wd, "layers": lambda i: ld[i % len(ld)]}
        self.mt, self.md = OracleGemma(st, wt, "fp32"), OracleGemma(sd, wd, "fp32")
        self.rng = np.random.default_rng(0)
        self.n = prompt_len
        nb = (prompt_len + (steps + 4) * (k + 1) + 32) // 16 + 2
        self.table = np.arange(nb, dtype=np.int32)[None]
        self.pt, self.pd = new_pages(st, nb, 16), new_pages(sd, nb, 16)
        prompt = self.rng.integers(0, 256000, prompt_len)[None]
        self.mt.forward(prompt, self.pt, self.table, [0], with_head=False)
        self.md.forward(prompt, self.pd, self.table, [0], with_head=False)

    def step(self) -> None:
        """One speculative step at full depth (random token ids: acceptance does not change the
        arithmetic of a step, only how many tokens it emits)."""
        import numpy as np

        toks = self.rng.integers(0, 256000, self.k + 1)
        for i in range(self.k):
            lg = self.md.forward(np.array([[toks[i]]]), self.pd, self.table, [self.n + i])
            int(np.argmax(lg[0, -1]))
        self.mt.forward(toks[None], self.pt, self.table, [self.n])
        self.n += 1

    def describe(self, tokens_per_step: float, threads: int) -> str:
        return (f"numpy oracle (port), fp32, full depth: {self.k} one-token Gemma-2B forwards (18 layers + LM head) "
                f"+ one Gemma-7B forward over {self.k + 1} tokens (28 layers + LM head) per step, after a "
                f"128-token prompt; layers cycle through {self.sample_layers[0]} / {self.sample_layers[1]} "
                f"distinct weight sets; {threads} BLAS threads; {tokens_per_step:.2f} tokens per step")


def run_reference(args):
    """--impl reference: the CPU restatement of the path (rank 0 only), one full-depth step per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    import numpy as np

    pipe = CpuPipeline(args.k, args.prompt_len, steps=args.warmup + args.steps)
    for _ in range(args.warmup):
        pipe.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        pipe.step()
        times.append(time.perf_counter() - t0)
    # random-init draft and target disagree, so one token (the recovery token) per step
    tokens_per_step = 1.0
    total_s = float(np.sum(times))
    value = tokens_per_step * args.steps / total_s
    desc = pipe.describe(tokens_per_step, threads) + f"; {args.steps} timed steps"
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * total_s / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": args.prompt_len, "k": args.k,
                       "parallelism": "cpu",
                       "l2": "host DRAM: the fp32 layer weights far exceed the CPU caches"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "threads": threads,
                             "cpu_count": os.cpu_count(), "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU leg
def _paired(w, args):
    """--qk-pairs: store q/k rows as rotation pairs, so RoPE and the K/V write run in the QKV epilogue."""
    return w.pair_qk_rows() if args.qk_pairs else w


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
    tp_parity = None
    if tp:
        from ssd_b200.runtime.tensor_parallel import TPComm, shard_weights, tp_selfcheck

        # Before the timed run: the sharded path's consistency checks on this run's GPUs
        # (bit-identical logits on every rank, sharded vs unsharded forward within the bf16
        # tolerance, sharded SD == sharded AR); any failure ends the run with a non-zero status.
        def gather(t):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            return parts

        tp_parity = tp_selfcheck(gather, device=dev)
        flag = torch.tensor([1 if tp_parity["ok"] else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        tp_parity = {k: v for k, v in tp_parity.items() if k != "ar"}
        tp_parity["ok_all_ranks"] = bool(flag.item())

        # every rank draws the same full weights from the seed and keeps its shard
        target = shard_weights(_paired(GemmaWeights.random(st_, seed=1000), args), rank, world)
        draft = shard_weights(_paired(GemmaWeights.random(sd_, seed=2000), args), rank, world)
        torch.cuda.empty_cache()
        comm = TPComm(heap_bytes=192 << 20, max_m=64, max_n=max(st_.d_model, sd_.d_model))
        rng = np.random.default_rng(0)
    else:
        target = _paired(GemmaWeights.random(st_, seed=1000 + rank), args)
        draft = _paired(GemmaWeights.random(sd_, seed=2000 + rank), args)
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
    clocks = ClockSampler(local, enabled=(rank == 0))
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
    n_prof = max(8, min(args.steps, 32))
    for _ in range(n_prof):
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

    status_all = 0
    if comm is not None:
        torch.cuda.synchronize()
        st_t = torch.tensor([comm.status()], dtype=torch.int32, device=dev)
        dist.all_reduce(st_t, op=dist.ReduceOp.MAX)
        status_all = int(st_t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            threads = cpu_threads()
            pipe = CpuPipeline(k, args.prompt_len, target.to_canonical(layers=2), draft.to_canonical(layers=1),
                               steps=9)
            pipe.step()
            t0 = time.perf_counter()
            n_cpu = 8
            for _ in range(n_cpu):
                pipe.step()
            step_s = (time.perf_counter() - t0) / n_cpu
            tps = tokens / args.steps
            cpu = {"value": tps / step_s, "unit": "tokens/s", "cores": threads, "threads": threads,
                   "cpu_count": os.cpu_count(), "kind": "port",
                   "sample": pipe.describe(tps, threads) + f"; {n_cpu} timed steps after one warm-up step "
                             f"(tokens per step taken from the GPU run)"}
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
                         # the events between launches break the programmatic-dependent-launch overlap
                         # of neighbouring kernels, so this window's launches run slower than in the
                         # timed (un-instrumented) verify step: achieved is a lower bound.  The timed
                         # verify step, attention and acceptance included, is verify_step_us.
                         "instrumented_proj_us_per_verify": 1000.0 * proj_ms / n_prof,
                         "uninstrumented_verify_step_us": verify_us,
                         "per_launch_bytes": proj_bytes / max(n_launch, 1), "per_kind": per_kind},
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": 16 * 4 + 8 * 4,
                    "d2h_bytes_per_step": 2 * 4 + (k + 1) * 4, "new_tokens": len(out),
                    "api": "SpeculativeDecoder.generate(prompt list) -> token list"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if tp_parity is not None:
            line["tp_parity"] = tp_parity
            line["tp_status_all_ranks"] = status_all
        print(json.dumps(line), flush=True)
    failed = (tp_parity is not None and not tp_parity["ok_all_ranks"]) or status_all != 0
    if failed:
        print(f"rank {rank}: tensor-parallel check failed (parity ok={tp_parity and tp_parity['ok_all_ranks']}, "
              f"collective status {status_all})", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    if failed:
        sys.exit(1)


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
    clocks = ClockSampler(local, enabled=(rank == 0))
    clocks.start()
    e0.record(stream)
    tokens = 0
    verify_ms = []
    ctx_sum = 0.0
    accepted = 0
    for _ in range(args.steps):
        ctx_sum += float(dec.t.n.sum())
        new = dec.step()
        tokens += sum(len(x) for x in new)
        accepted += int(dec.last_accept.sum())
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
    # FLOPs per step on this rank: 2 per weight element per token row (verify: B*(k+1) rows,
    # each draft forward: B rows), plus q.k and p.v over the context (4 * ctx * Hq * D per row, layer)
    def model_flops(sh, vocab_rows, rows):
        params = sh.layer_weight_bytes() // 2 * sh.num_layers + vocab_rows * sh.d_model
        attn = 4.0 * mean_ctx * sh.num_heads * sh.head_dim * sh.num_layers
        return rows * (2.0 * params + attn)
    step_flops = model_flops(lt, st_.vocab // world, B * (k + 1)) + k * model_flops(ld, sd_.vocab // world, B)
    try:
        tflops_peak = float(json.loads(PEAKS.read_text())["bf16_tflops_sustained"])
        tflops_kind = "measured (sustained)"
    except Exception:
        tflops_peak, tflops_kind = 1400.0, "fallback (sustained)"
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
            "tokens_per_step": tokens / args.steps, "accept_rate": accepted / (args.steps * B * k),
            "verify_ms": statistics.mean(verify_ms),
            "step_bytes_per_rank": step_bytes, "step_hbm_gbs": step_bytes / step_s / 1e9,
            "step_roofline_frac": step_bytes / step_s / 1e9 / hbm, "peak_kind": kind,
            "step_flops_per_rank": step_flops, "step_tflops": step_flops / step_s / 1e12,
            "step_flop_frac": step_flops / step_s / 1e12 / tflops_peak, "flop_peak_kind": tflops_kind,
            "clocks": clk,
        }), flush=True)
    if world > 1:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def run_ssd(args):
    """Async ssd mode (speculation cache, fan-out per accepted length) with the Gemma-7B target
    tensor-parallel over GPUs 0..T-1 and the Gemma-2B draft on GPU T, through the public API
    (``LLM.generate``, one process, one thread per target GPU).  The step is a host protocol (draft
    worker thread, queues), so ``value`` is wall clock around ``generate`` (prefill included);
    ``verify_step_us`` is the CUDA-event time of the target's verify forward + acceptance on
    rank 0."""
    import numpy as np
    import torch

    from ssd_b200 import LLM, DecodeMode, SamplingParams, SSDConfig

    T, k = args.tp, args.k
    ngpu = torch.cuda.device_count()
    if ngpu < T:
        print(json.dumps({"mode": "ssd", "unavailable": f"needs {T} GPUs, {ngpu} visible"}), flush=True)
        return
    cfg = SSDConfig(mode=DecodeMode.SSD, speculate_k=k, fan_out_list=(args.fanout,) * (k + 1),
                    target_model_path="gemma-7b", draft_model_path="gemma-2b", use_toy_model=False,
                    tensor_parallel_size=T, max_model_len=args.prompt_len + args.new_tokens + 64, seed=1000,
                    draft_device=f"cuda:{T}" if ngpu > T else "cuda:0")
    llm = LLM(cfg)
    eng = llm._engine
    rng = np.random.default_rng(0)
    prompt = [int(x) for x in rng.integers(0, 256000, args.prompt_len)]
    llm.generate([prompt[:64]], SamplingParams(max_new_tokens=2 * (k + 1)))  # warm-up
    clocks = ClockSampler(0)
    clocks.start()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out, m = llm.generate([prompt], SamplingParams(max_new_tokens=args.new_tokens))
    t1 = time.perf_counter()
    clk = clocks.stop()
    llm.shutdown()
    n_tok = len(out[0])
    from ssd_b200.models.gemma import PRESETS
    from ssd_b200.runtime.tensor_parallel import shard_layout

    st_, _ = shard_layout(PRESETS["gemma-7b"], 0, T)  # one rank's shard
    vocab = st_.vocab
    steps = m.steps
    verify_us = 1000.0 * statistics.mean(s.verify_device_ms for s in steps)
    draft_ms = statistics.mean(s.draft_step_ms for s in steps)
    mean_ctx = args.prompt_len + n_tok / 2
    wbytes = st_.layer_weight_bytes() * st_.num_layers + (vocab // T) * st_.d_model * 2
    vbytes = wbytes + st_.kv_bytes_per_token() * mean_ctx + (k + 1) * vocab * 4
    hbm, kind = peaks()
    acc = sum(a * c for a, c in m.accept_histogram.items()) / max(1, sum(m.accept_histogram.values()))
    print(json.dumps({
        "metric": "Gemma-7B/2B ssd tokens/sec, target TP + draft GPU; verify-step µs; HBM GB/s",
        "value": n_tok / (t1 - t0), "unit": "tokens/s", "mode": "ssd", "n_gpus": T + (1 if eng.draft_device.index >= T else 0),
        "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (random-init weights, random prompt ids)",
        "config": {"workload": f"gemma-7b target (TP{T}) + gemma-2b draft on {eng.draft_device}, async ssd, "
                               f"fan-out {args.fanout}, k={k}, prompt {args.prompt_len}, {args.new_tokens} new",
                   "parallelism": f"tp{T}+draft", "fan_out_list": list(cfg.fan_out_list)},
        "steps": len(steps), "ms_per_step": 1000.0 * (t1 - t0) / max(1, len(steps)),
        "verify_step_us": verify_us, "verify_hbm_gbs_per_rank": vbytes / (verify_us / 1e6) / 1e9,
        "verify_roofline_frac": vbytes / (verify_us / 1e6) / 1e9 / hbm, "peak_kind": kind,
        "draft_wait_ms_per_step": draft_ms, "accepted_per_step": acc, "cache_hit_rate": m.cache_hit_rate,
        "tokens_per_step": m.accepted_per_step, "ttft_s": m.ttft_s,
        "e2e": {"value": n_tok / (t1 - t0), "unit": "tokens/s", "api": "LLM.generate(prompt list) -> token lists",
                "h2d_bytes_per_step": 4 * (k + 1) * T, "d2h_bytes_per_step": 8 * T + 4 * k},
        "clocks": clk,
    }), flush=True)


def main():
    args = parse()
    if args.mode == "ssd" and args.impl == "ours":
        run_ssd(args)
        return
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
