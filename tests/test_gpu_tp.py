"""The fused tensor-parallel projections and the sharded forward on ONE GPU (a group of one).

With ``world == 1`` the collective kernels run their whole protocol -- pushes into
the heap, per-tile flags, the device sequence word, parity buffers, the exit
counter -- against the local heap, and must reproduce the plain projections bit
for bit.  The multi-GPU runs are in ``test_gpu_tp_multi.py``.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm(cuda):
    from ssd_b200.runtime.tensor_parallel import TPComm

    c = TPComm(heap_bytes=64 << 20, max_m=256, max_n=4096, device=cuda)
    yield c
    c.close()


@pytest.mark.parametrize("m,n,k", [(5, 3072, 4096), (5, 3072, 3072), (1, 256, 128), (37, 384, 512),
                                   (200, 1024, 1024), (16, 3072, 24576)])
def test_allreduce_group_of_one_equals_residual(comm, cuda, m, n, k):
    from ssd_b200.kernels.ops import linear, linear_allreduce

    g = torch.Generator(device=cuda).manual_seed(m * 7 + n + k)
    x = torch.randn((m, k), generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device=cuda) / k ** 0.5).to(torch.bfloat16)
    y0 = torch.randn((m, n), generator=g, device=cuda).to(torch.bfloat16)
    want = linear(x, w, "residual", out=y0.clone())
    c0 = comm.tile_counts(1)[0]
    for rep in range(3):  # both parities, repeated use of the same flags
        got = linear_allreduce(x, w, y0.clone(), comm)
        torch.cuda.synchronize()
        assert torch.equal(got, want), rep
    assert comm.tile_counts(1)[0] == (c0 + 3) & 0xFFFFFFFF
    assert comm.status() == 0


@pytest.mark.parametrize("m,n,k", [(5, 2048, 256), (1, 32000, 3072), (40, 1000, 512)])
def test_allgather_group_of_one_equals_store_f32(comm, cuda, m, n, k):
    from ssd_b200.kernels.ops import linear, linear_allgather

    g = torch.Generator(device=cuda).manual_seed(n + k)
    x = torch.randn((m, k), generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device=cuda) / k ** 0.5).to(torch.bfloat16)
    want = linear(x, w, "store_f32")
    top = comm._top
    y = comm.alloc((m, n), torch.float32)
    c0 = comm.tile_counts(1)[0]
    linear_allgather(x, w, y, comm)
    linear_allgather(x, w, y, comm)
    torch.cuda.synchronize()
    comm._top = top  # give the buffer back
    assert torch.equal(y, want)
    assert comm.tile_counts(1)[0] == (c0 + 2) & 0xFFFFFFFF and comm.status() == 0


def test_forward_with_group_of_one_equals_plain(comm, cuda):
    from ssd_b200.kernels.kv_cache import KVCacheState
    from ssd_b200.models.gemma import PRESETS, GemmaRunner, GemmaWeights

    s = PRESETS["tp-target"]
    w = GemmaWeights.random(s, seed=11, device=cuda, max_pos=512)
    toks = torch.randint(0, s.vocab, (1, 21), device=cuda, dtype=torch.int32)
    outs = []
    top = comm._top
    for use in (False, True):
        cache = KVCacheState.allocate(s.num_layers, 8, 16, s.num_kv_heads, s.head_dim, torch.bfloat16, cuda)
        table = torch.arange(8, dtype=torch.int32, device=cuda)[None]
        r = GemmaRunner(w, 1, 64, 128, comm=comm if use else None)
        lg = comm.alloc((1, 21, s.vocab)) if use else torch.empty((1, 21, s.vocab), device=cuda)
        r.forward(toks, torch.zeros(1, dtype=torch.int32, device=cuda), cache.pages, table, lg)
        torch.cuda.synchronize()
        outs.append(lg.clone())
    comm._top = top
    assert torch.equal(outs[0], outs[1])
    assert comm.status() == 0


def test_speculative_decoder_with_group_of_one(comm, cuda):
    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.runtime.speculative import GreedyDecoder, SpeculativeDecoder

    t = GemmaWeights.random(PRESETS["tp-target"], seed=21, device=cuda, max_pos=512)
    prompt = list(range(100, 140))
    top = comm._top
    ar = GreedyDecoder(t, max_seq_len=256).generate(prompt, 24)
    ar_c = GreedyDecoder(t, max_seq_len=256, comm=comm).generate(prompt, 24)
    # self-draft: every draft accepted; graphs replayed after the first eager steps
    sd = SpeculativeDecoder(t, t, k=4, max_seq_len=256, comm=comm)
    out, _ = sd.generate(prompt, 24)
    comm._top = top
    assert ar == ar_c == out
    assert comm.status() == 0
