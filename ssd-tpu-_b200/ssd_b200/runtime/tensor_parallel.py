"""Tensor parallelism over NVLink: symmetric heaps, weight sharding, the comm handle.

One process per GPU (``torch.distributed`` only carries the 64-byte IPC handles
at set-up).  Each rank allocates one device "heap" of the same size and maps
every peer's heap into its own address space (``ssd_ipc_export`` /
``ssd_ipc_import``); the heap holds the control block of the fused collectives,
the all-reduce receive area, and buffers that peers write into (the logits the
vocab-parallel LM head all-gathers), carved at identical offsets on every rank.

Sharding of a Gemma layer over ``world`` ranks (Megatron-style):

* q heads ``[r*Hq/w, (r+1)*Hq/w)``; KV heads the matching block when
  ``Hkv % w == 0``, the single KV head replicated for multi-query attention;
* ``w_qkv`` / ``w_gate_up`` row blocks (column-parallel, the folded RMSNorm
  needs the full residual row, which every rank holds), ``w_o`` / ``w_down``
  column blocks (row-parallel: partial products all-reduced in the projection
  kernel, ``ssd_linear_allreduce``);
* the embedding table replicated; rows ``[r*V/w, (r+1)*V/w)`` are rank r's block
  of the tied LM head (``ssd_linear_allgather``).

The reference shards with XLA GSPMD (jax_ssd/models/sharding.py:10-31); there
is no tensor-parallel arithmetic there to match, so a sharded forward is
checked against the unsharded oracle within the bf16 tolerance.
"""

from __future__ import annotations

import ctypes as C

import torch

from .._lib import SSD_ALLREDUCE_ALL_TO_ALL, SSD_ALLREDUCE_AUTO, SSD_ALLREDUCE_OWNER, SSD_MAX_TP, CommC, check, lib


class TPComm:
    """The ``ssd_comm`` handle of one rank plus a bump allocator over its heap.

    ``alloc`` must be called with the same sizes in the same order on every
    rank (buffers are symmetric by construction).  ``world == 1`` needs no
    process group: the collective kernels then run against the local heap only
    (used to exercise the fused path on one GPU).
    """

    def __init__(self, heap_bytes: int = 256 << 20, max_m: int = 256, max_n: int = 8192, group=None,
                 device=None):
        import torch.distributed as dist

        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        if not 1 <= self.world <= SSD_MAX_TP:
            raise ValueError(f"tensor parallelism supports 1..{SSD_MAX_TP} ranks, got {self.world}")
        L = lib()
        self.ctrl_bytes = int(L.ssd_comm_ctrl_bytes())
        self.recv_bytes = int(L.ssd_comm_recv_bytes(self.world, max_m, max_n))
        fixed = self.ctrl_bytes + self.recv_bytes
        heap_bytes = max(heap_bytes, fixed + (1 << 20))
        self.heap = torch.zeros(heap_bytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        self._top = fixed
        self._imported: list[tuple[int, int]] = []
        self.heap_bytes, self.max_m, self.max_n = heap_bytes, max_m, max_n
        peers: list[int] = []
        if self.world > 1:
            handle = (C.c_char * 64)()
            off = C.c_size_t(0)
            check(L.ssd_ipc_export(self.heap.data_ptr(), handle, C.byref(off)), "ssd_ipc_export")
            mine = (bytes(handle), int(off.value), self.device.index)
            everyone: list = [None] * self.world
            dist.all_gather_object(everyone, mine, group=group)
            if len({e[2] for e in everyone}) != self.world:
                raise ValueError("tensor-parallel ranks must sit on distinct GPUs")
            for r, (h, o, _) in enumerate(everyone):
                if r == self.rank:
                    peers.append(self.heap.data_ptr())
                    continue
                p = C.c_void_p()
                hb = (C.c_char * 64).from_buffer_copy(h)
                check(L.ssd_ipc_import(hb, o, C.byref(p)), "ssd_ipc_import")
                peers.append(int(p.value))
                self._imported.append((int(p.value), o))
            dist.barrier(group=group)
        else:
            peers = [self.heap.data_ptr()]
        self._bind(peers)

    def _bind(self, peers: list[int]) -> None:
        c = CommC()
        c.rank, c.world = self.rank, self.world
        for r in range(SSD_MAX_TP):
            c.heaps[r] = peers[r] if r < self.world else None
        c.heap_bytes = self.heap_bytes
        c.ctrl_offset = 0
        c.recv_offset = self.ctrl_bytes
        c.recv_bytes = self.recv_bytes
        c.recv_rows, c.recv_tiles = self.max_m, (self.max_n + 127) // 128
        c.allreduce_form = SSD_ALLREDUCE_AUTO
        self.cstruct = c

    def set_allreduce_form(self, form: int) -> None:
        """SSD_ALLREDUCE_AUTO / _ALL_TO_ALL / _OWNER for the following all-reduces (every rank alike)."""
        self.cstruct.allreduce_form = int(form)

    def alloc(self, shape, dtype=torch.float32) -> torch.Tensor:
        """A symmetric buffer (same heap offset on every rank), 256-byte aligned, zero-filled."""
        n = 1
        for d in shape:
            n *= int(d)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        start = (self._top + 255) & ~255
        if start + nbytes > self.heap.numel():
            raise MemoryError(f"symmetric heap exhausted ({self.heap.numel()} bytes)")
        self._top = start + nbytes
        return self.heap[start:start + nbytes].view(dtype).view(*shape)

    def mark(self) -> int:
        """The allocator's current top; ``release(mark)`` frees everything allocated after it."""
        return self._top

    def release(self, mark: int) -> None:
        """Free the buffers allocated since ``mark`` (same call on every rank; their tensors must
        no longer be used)."""
        if not 0 <= mark <= self._top:
            raise ValueError("release() needs a mark taken from this heap")
        self._top = mark

    def status(self) -> int:
        """Word 2 of the control block: 0, or SSD_ERR_TIMEOUT after a peer wait gave up."""
        return int(self.heap[8:12].view(torch.int32).item())

    def tile_counts(self, n: int = 8) -> list[int]:
        """Collectives finished so far for output tiles 0..n-1 (device counters)."""
        off = 256
        return [int(v) & 0xFFFFFFFF for v in self.heap[off:off + 4 * n].view(torch.int32).tolist()]

    def close(self) -> None:
        L = lib()
        for p, o in self._imported:
            L.ssd_ipc_close(p, o)
        self._imported = []


def shard_layout(shape, rank: int, world: int):
    """Per-rank shape and the index blocks of rank ``rank`` (host arithmetic only)."""
    from ..models.gemma import GemmaShape

    s = shape
    if s.num_heads % world or s.ffn % world or s.vocab % world:
        raise ValueError(f"{s} does not shard over {world} ranks")
    if s.num_kv_heads % world == 0:
        hkv_l, kv0 = s.num_kv_heads // world, rank * (s.num_kv_heads // world)
    elif s.num_kv_heads == 1:
        hkv_l, kv0 = 1, 0  # multi-query: the single KV head is replicated
    else:
        raise ValueError(f"{s.num_kv_heads} KV heads do not shard over {world} ranks")
    hq_l, f_l = s.num_heads // world, s.ffn // world
    local = GemmaShape(s.num_layers, s.d_model, hq_l, hkv_l, s.head_dim, f_l, s.vocab, s.eps, s.rope_theta)
    return local, {"q": (rank * hq_l, hq_l), "kv": (kv0, hkv_l), "ffn": (rank * f_l, f_l),
                   "vocab": (rank * (s.vocab // world), s.vocab // world)}


def shard_weights(full, rank: int, world: int):
    """Rank ``rank``'s shard of a ``GemmaWeights`` (see the module docstring)."""
    from ..models.gemma import GemmaWeights

    s = full.shape
    local, blk = shard_layout(s, rank, world)
    D = s.head_dim
    q0, nq = blk["q"]
    k0, nk = blk["kv"]
    f0, nf = blk["ffn"]
    hq_rows, hkv_rows = s.num_heads * D, s.num_kv_heads * D
    w = GemmaWeights(local, full.dtype, full.device, full.max_pos)
    w.embed = full.embed  # replicated (shared storage)
    w.final_norm = full.final_norm
    for l in range(s.num_layers):
        qkv = full.w_qkv[l]
        w.w_qkv[l].copy_(torch.cat([
            qkv[q0 * D:(q0 + nq) * D],
            qkv[hq_rows + k0 * D:hq_rows + (k0 + nk) * D],
            qkv[hq_rows + hkv_rows + k0 * D:hq_rows + hkv_rows + (k0 + nk) * D]], 0))
        w.w_o[l].copy_(full.w_o[l][:, q0 * D:(q0 + nq) * D])
        w.w_gate_up[l].copy_(full.w_gate_up[l][2 * f0:2 * (f0 + nf)])
        w.w_down[l].copy_(full.w_down[l][:, f0:f0 + nf])
        w.attn_norm[l] = full.attn_norm[l]
        w.mlp_norm[l] = full.mlp_norm[l]
    w.rope_cos, w.rope_sin = full.rope_cos, full.rope_sin
    w.tp_rank, w.tp_world = rank, world
    w.qk_pairs = full.qk_pairs  # head blocks of rotation-paired rows stay paired
    return w


def tp_selfcheck(all_gather, device=None, heap_bytes: int = 64 << 20) -> dict:
    """Consistency checks of the sharded path, run by every rank of an initialised process group.

    On the small bf16 ``tp-target`` / ``tp-draft`` presets (seeded weights, every projection on the
    tcgen05 path at 1..8 ranks):

    * ``ranks_identical``: every rank holds bit-identical logits after the sharded forward (the
      collectives add the ranks' partials in rank order on every rank);
    * ``max_diff`` / ``scale``: the sharded forward against the unsharded forward of the same
      weights on this GPU, |difference| <= 2e-2 * max(max|logit|, 1) (bf16 rounding of the partial
      sums is the only difference);
    * ``sd_equals_ar``: greedy speculative decoding on the sharded pair reproduces the sharded
      target's AR stream (``self_sd_equals_ar``: with the target as its own draft, every draft is
      accepted and the stream is still the AR stream);
    * ``allreduce_exact``: ``linear_allreduce`` at 5, 40 and 224 rows, in each of its forms (automatic,
      all-to-all, via the tile's owner), equals, bit for bit, bf16(y + bf16(sum of the ranks' fp32
      partials in rank order)), the partials being each rank's plain projection of its shard.

    ``all_gather(tensor) -> list[tensor]`` gathers a CUDA tensor from every rank.  Returns a dict;
    ``ok`` is the conjunction of the checks and of a zero collective status.
    """
    from ..kernels.kv_cache import KVCacheState
    from ..models.gemma import PRESETS, GemmaRunner, GemmaWeights
    from .speculative import GreedyDecoder, SpeculativeDecoder

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    comm = TPComm(heap_bytes=heap_bytes, max_m=256, max_n=4096, device=dev)
    rank, world = comm.rank, comm.world
    out: dict = {"world": world}
    ok = True
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
            torch.cuda.synchronize(dev)
            res[tag] = lg.clone()
        diff = (res["tp"] - res["full"]).abs().max().item()
        scale = res["full"].abs().max().item()
        gathered = all_gather(res["tp"])
        same = all(torch.equal(g, gathered[0]) for g in gathered)
        good = same and diff <= 2e-2 * max(scale, 1.0)
        out[name] = {"max_diff": diff, "scale": scale, "ranks_identical": same, "ok": good}
        ok = ok and good
    from ..kernels.ops import linear, linear_allreduce

    exact = {}
    for m in (5, 40, 224):
        g = torch.Generator(device=dev).manual_seed(1000 * m + rank)
        x = torch.randn((m, 256), generator=g, device=dev).bfloat16()
        w = (torch.randn((4096, 256), generator=g, device=dev) / 16).bfloat16()
        y0 = (torch.arange(m * 4096, device=dev, dtype=torch.float32).reshape(m, 4096) % 7 - 3).bfloat16()
        part = linear(x, w, "store_f32", ws_key="tp_selfcheck")
        torch.cuda.synchronize(dev)
        parts = [pr.cpu() for pr in all_gather(part)]
        acc = torch.zeros_like(parts[0])
        for pr in parts:  # rank order, one fp32 add at a time
            acc = acc + pr
        want = (y0.float().cpu() + acc.bfloat16().float()).bfloat16()
        for form, tag in ((SSD_ALLREDUCE_AUTO, "auto"), (SSD_ALLREDUCE_ALL_TO_ALL, "all_to_all"),
                          (SSD_ALLREDUCE_OWNER, "owner")):
            comm.set_allreduce_form(form)
            got = linear_allreduce(x, w, y0.clone(), comm, ws_key="tp_selfcheck")
            torch.cuda.synchronize(dev)
            exact[f"{tag}_m{m}"] = bool(torch.equal(got.cpu(), want))
    comm.set_allreduce_form(SSD_ALLREDUCE_AUTO)
    out["allreduce_exact"] = exact
    ok = ok and all(exact.values())
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
    torch.cuda.synchronize(dev)
    out["status"] = comm.status()
    ars = all_gather(torch.tensor(ar, dtype=torch.int32, device=dev))
    out["ar_identical_across_ranks"] = all(torch.equal(a, ars[0]) for a in ars)
    out["ok"] = bool(ok and out["sd_equals_ar"] and out["self_sd_equals_ar"] and out["status"] == 0
                     and out["ar_identical_across_ranks"] and st["steps"] < 32)
    comm.close()
    return out
