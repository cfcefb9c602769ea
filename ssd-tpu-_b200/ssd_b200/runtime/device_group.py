"""Several GPUs driven by one process: one host thread per GPU.

The reference is a single controller that places arrays on device meshes
(connect/mesh_allocator.py:64-117, jax_ssd/models/sharding.py:10-31).  The
tensor-parallel kernels of this package are SPMD instead: every rank issues
the same launches on its own GPU and the fused collectives meet over NVLink.
``DeviceGroup`` runs that SPMD program inside one process -- one worker thread
per GPU, each with its GPU current -- so ``LLM`` keeps the reference's
single-process API while the target runs tensor-parallel.

``run(fn)`` executes ``fn(rank)`` on every worker at once and returns the
results in rank order; the first exception raised on any rank is re-raised in
the caller after all ranks have returned (a rank whose peers stopped issuing
work ends its collective waits with a timeout status instead of hanging).
Kernel launches and graph replays release the GIL, so the ranks' launches
interleave freely.
"""

from __future__ import annotations

import queue
import threading

import torch


class DeviceGroup:
    def __init__(self, devices) -> None:
        self.devices = [torch.device(d) if not isinstance(d, int) else torch.device("cuda", d) for d in devices]
        if not self.devices:
            raise ValueError("a device group needs at least one GPU")
        self._queues: list[queue.Queue] = [queue.Queue() for _ in self.devices]
        self._threads = [threading.Thread(target=self._loop, args=(r,), daemon=True)
                         for r in range(len(self.devices))]
        for t in self._threads:
            t.start()

    @property
    def world(self) -> int:
        return len(self.devices)

    def _loop(self, rank: int) -> None:
        torch.cuda.set_device(self.devices[rank])
        while True:
            item = self._queues[rank].get()
            if item is None:
                return
            fn, out, done = item
            try:
                out[rank] = (True, fn(rank))
            except BaseException as exc:  # handed back to the caller of run()
                out[rank] = (False, exc)
            finally:
                done.release()

    def run(self, fn):
        """``[fn(0), ..., fn(world - 1)]``, each on its own GPU's thread, concurrently."""
        out: list = [None] * self.world
        done = threading.Semaphore(0)
        for q in self._queues:
            q.put((fn, out, done))
        for _ in range(self.world):
            done.acquire()
        for ok, val in out:
            if not ok:
                raise val
        return [val for _, val in out]

    def close(self) -> None:
        for q in self._queues:
            q.put(None)
        for t in self._threads:
            t.join(timeout=30)
