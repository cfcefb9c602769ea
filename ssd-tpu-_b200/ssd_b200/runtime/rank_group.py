"""The target's tensor-parallel group behind the single-process ``LLM`` API: one worker process per GPU.

The reference is a single controller that places arrays on device meshes
(connect/mesh_allocator.py:64-117, jax_ssd/models/sharding.py:10-31).  The
tensor-parallel kernels of this package are SPMD instead: every rank issues the
same launches on its own GPU and the fused collectives meet over NVLink, each
waiting (boundedly) for its peers.  Ranks therefore must never wait on one
another on the host, which rules out threads of one Python process (a torch
call that synchronises while holding the interpreter lock would stop the other
ranks from launching).  ``RankGroup`` spawns one process per GPU instead; the
ranks form a ``torch.distributed`` (gloo) group only to exchange the 64-byte
CUDA IPC handles of their symmetric heaps (``TPComm``), and the engine drives
them with small commands over pipes: every command runs on every rank and
returns every rank's (picklable) result.

``RankState`` is what one rank holds -- its weight shards, its ``TPComm`` and
the decoders -- and its methods are the commands.  With one GPU the engine
keeps a ``RankState`` in its own process (``LocalRank``), so both cases share
one code path.
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import socket
import traceback

import torch


class RankState:
    """One rank's share of the engine (weights, comm, decoders); its methods are the commands."""

    def __init__(self, cfg: dict, rank: int, world: int, device_index: int) -> None:
        from ..models.gemma import PRESETS
        from ..models.model_loader import default_preset, load_sharded_weights, load_weights

        self.cfg = cfg
        self.rank, self.world = rank, world
        self.dev = torch.device("cuda", device_index)
        torch.cuda.set_device(self.dev)
        use_toy = cfg["use_toy_model"]
        tpath, dpath = cfg["target_model_path"], cfg["draft_model_path"]
        self.comm = None
        if world == 1:
            self.target_w = load_weights(tpath, use_toy=use_toy, seed=cfg["seed"], role="target", device=self.dev)
        else:
            from .tensor_parallel import TPComm

            self.target_w = load_sharded_weights(tpath, rank, world, use_toy=use_toy, seed=cfg["seed"],
                                                 role="target", device=self.dev)
            pre = lambda p, role: p if p in PRESETS else default_preset(role, use_toy)  # noqa: E731
            d_model = max(PRESETS[pre(tpath, "target")].d_model, PRESETS[pre(dpath, "draft")].d_model)
            self.comm = TPComm(heap_bytes=cfg.get("heap_bytes", 512 << 20), max_m=256, max_n=d_model,
                               device=self.dev)
        self.draft_w = None
        if cfg["local_draft"]:  # sd / ar modes: the draft runs on the target's GPUs (sharded when world > 1)
            if world == 1:
                self.draft_w = load_weights(dpath, use_toy=use_toy, seed=cfg["draft_seed"], role="draft",
                                            device=self.dev)
            else:
                self.draft_w = load_sharded_weights(dpath, rank, world, use_toy=use_toy, seed=cfg["draft_seed"],
                                                    role="draft", device=self.dev)
        self.target = None  # GemmaAdapter of the ssd loop
        self.dec = None
        self._mark = None
        if cfg.get("target_adapter"):
            self._adapter()  # its heap buffers are allocated before any generate call's mark

    # ------------------------------------------------------------ buffers
    def begin(self) -> None:
        """Start of a generate call: later symmetric-heap buffers are released by ``end``."""
        self._mark = self.comm.mark() if self.comm is not None else None

    def end(self) -> int:
        """End of a generate call: drop its decoders, free their heap buffers; the collective status."""
        torch.cuda.current_stream().synchronize()
        self.dec = None
        status = 0
        if self.comm is not None:
            status = self.comm.status()
            if self._mark is not None:
                self.comm.release(self._mark)
        return status

    # ------------------------------------------------------------ ar
    def ar_generate(self, prompt: list[int], max_new: int, max_len: int, block_size: int) -> list[int]:
        from .speculative import GreedyDecoder

        return GreedyDecoder(self.target_w, max_seq_len=max_len, block_size=block_size,
                             comm=self.comm).generate(prompt, max_new)

    # ------------------------------------------------------------ sd, one sequence (graph-replayed step)
    def sd_start(self, prompt: list[int], k: int, max_len: int, block_size: int) -> int:
        from .speculative import SpeculativeDecoder

        self.dec = SpeculativeDecoder(self.target_w, self.draft_w, k=k, max_seq_len=max_len, block_size=block_size,
                                      comm=self.comm)
        return self.dec.start(prompt)

    def sd_step(self) -> tuple[list[int], float, int]:
        new = self.dec.step()
        return new, self.dec.last_verify_ms, int(self.dec.last_accept)

    # ------------------------------------------------------------ sd, batched rows (continuous batching)
    def batch_open(self, batch: int, k: int, max_len: int, block_size: int, temperature: float, top_p: float,
                   sampler_x: float, seed: int) -> None:
        from .batched import BatchedSpeculativeDecoder

        self.dec = BatchedSpeculativeDecoder(self.target_w, self.draft_w, batch=batch, k=k, max_seq_len=max_len,
                                             block_size=block_size, temperature=temperature, top_p=top_p,
                                             sampler_x=sampler_x, seed=seed, comm=self.comm)

    def batch_admit(self, placed: list[tuple[int, list[int]]]) -> list[int]:
        return [self.dec.admit(slot, prompt) for slot, prompt in placed]

    def batch_park(self, slot: int) -> None:
        self.dec.park(slot)

    def batch_step(self) -> tuple[list[list[int]], float, list[int]]:
        new = self.dec.step()
        return new, self.dec.last_verify_ms, [int(a) for a in self.dec.last_accept]

    # ------------------------------------------------------------ ssd: the target side of the async protocol
    def _adapter(self):
        if self.target is None:
            from ..models.gemma_adapter import GemmaAdapter

            self.target = GemmaAdapter(self.target_w, max_model_len=self.cfg["max_model_len"], name="target",
                                       comm=self.comm)
        return self.target

    def target_prefill(self, prompt: list[int]) -> int:
        """Prefill the target; the greedy first token (argmax of the last prompt position)."""
        from ..algorithm.verify import argmax_rows

        lg = self._adapter().prefill(torch.tensor(prompt, dtype=torch.int32)).logits
        out = torch.empty(1, dtype=torch.int32, device=self.dev)
        argmax_rows(lg.contiguous(), out)
        return int(out.item())

    def target_verify(self, spec_kp1: list[int]) -> tuple[int, int, float]:
        """Verify forward over [recovery] + drafts and greedy acceptance: (accepted, recovery, device ms)."""
        from ..algorithm.verify import verify_greedy

        st = torch.cuda.current_stream()
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(st)
        toks = torch.tensor([spec_kp1], dtype=torch.int32, device=self.dev)
        vres = self._adapter().verify(toks)
        vout = verify_greedy(vres.logits, toks)
        ev[1].record(st)
        acc, rec = int(vout.accept_until[0]), int(vout.recovery_tokens[0])
        return acc, rec, ev[0].elapsed_time(ev[1])

    def target_commit(self, tokens: list[int]) -> None:
        self._adapter().commit_tokens(tokens)

    def close(self) -> None:
        torch.cuda.synchronize(self.dev)
        self.dec = None
        self.target = None
        if self.comm is not None:
            self.comm.close()


class LocalRank:
    """A one-GPU group: the ``RankState`` lives in the caller's process."""

    world = 1

    def __init__(self, cfg: dict, device_index: int) -> None:
        with torch.cuda.device(device_index):
            self.state = RankState(cfg, 0, 1, device_index)
        self.device_index = device_index

    def call(self, name: str, *args):
        with torch.cuda.device(self.device_index):
            return [getattr(self.state, name)(*args)]

    def close(self) -> None:
        self.state.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _resolve(path: str):
    import importlib

    mod, _, name = path.partition(":")
    return getattr(importlib.import_module(mod), name)


def _worker(rank: int, world: int, device_index: int, port: int, cfg: dict, conn, state_cls: str) -> None:
    try:
        import torch.distributed as dist

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        state = _resolve(state_cls)(cfg, rank, world, device_index)
        conn.send(("ok", None))
    except BaseException:
        conn.send(("err", traceback.format_exc()))
        return
    while True:
        try:
            msg = conn.recv()
        except EOFError:
            break
        if msg is None:
            break
        name, args = msg
        try:
            conn.send(("ok", getattr(state, name)(*args)))
        except BaseException:
            conn.send(("err", traceback.format_exc()))
    try:
        state.close()
        dist.destroy_process_group()
    except BaseException:
        pass


class RankGroup:
    """One spawned worker process per GPU of ``devices``, rank r on ``devices[r]``.

    ``state_cls`` ("module:Class") is what each worker builds as ``Class(cfg, rank, world, device)``;
    the engine uses ``RankState``.
    """

    def __init__(self, devices: list[int], cfg: dict,
                 state_cls: str = "ssd_b200.runtime.rank_group:RankState") -> None:
        ctx = mp.get_context("spawn")
        port = _free_port()
        self.world = len(devices)
        self._conns, self._procs = [], []
        for r, d in enumerate(devices):
            parent, child = ctx.Pipe()
            p = ctx.Process(target=_worker, args=(r, self.world, d, port, cfg, child, state_cls), daemon=True)
            p.start()
            self._conns.append(parent)
            self._procs.append(p)
        try:
            errors = [m for m in (self._recv(c) for c in self._conns) if m[0] != "ok"]
        except RuntimeError:
            self.close()
            raise
        if errors:
            self.close()
            raise RuntimeError("tensor-parallel rank failed to start:\n" + errors[0][1])

    @staticmethod
    def _recv(conn):
        try:
            return conn.recv()
        except EOFError:
            raise RuntimeError("a tensor-parallel rank process exited") from None

    def call(self, name: str, *args):
        """Run ``<state>.<name>(*args)`` on every rank; the results in rank order.  A rank that raises
        makes the call raise (with that rank's traceback) after every rank has answered."""
        for c in self._conns:
            c.send((name, args))
        out = [self._recv(c) for c in self._conns]
        bad = [m for m in out if m[0] != "ok"]
        if bad:
            raise RuntimeError(f"tensor-parallel rank failed in {name}:\n" + bad[0][1])
        return [m[1] for m in out]

    def close(self) -> None:
        for c in self._conns:
            try:
                c.send(None)
            except Exception:
                pass
        for p in self._procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
        self._conns, self._procs = [], []
