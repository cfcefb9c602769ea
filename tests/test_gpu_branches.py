"""Branch decoding for the async SSD fan-out: page fork + batched branch drafting.

* ``ssd_page_fork`` leaves tables, lengths, free list and ref counts exactly as
  the oracle's fork, and copies the partial trunk page's K/V rows;
* ``GemmaAdapter.draft_branches`` (forked trunk, batched forwards over the
  branch rows) drafts exactly what one ``draft_speculate`` per branch drafts.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("num_tokens", [40, 32, 7])
def test_page_fork_matches_oracle_and_copies_rows(cuda, num_tokens):
    from oracle.page_manager import OraclePageManager, OracleSeq, to_dense
    from ssd_b200.kernels.kv_cache import KVCacheState
    from ssd_b200.runtime.page_manager import PageManager

    bs, nb, n = 16, 40, 4
    pm = PageManager(bs, nb, max_seqs=1 + n, max_blocks_per_seq=8, device=cuda)
    cache = KVCacheState.allocate(2, nb, bs, 2, 64, dtype=torch.bfloat16, device=cuda)
    cache.pages.normal_()
    pm.allocate_rows(0, 1, torch.tensor([0], dtype=torch.int32, device=cuda),
                     torch.tensor([num_tokens + 9], dtype=torch.int32, device=cuda), None)
    ok = pm.fork_rows(0, 1, n, num_tokens, cache)
    torch.cuda.synchronize()
    # oracle
    opm = OraclePageManager(block_size=bs, num_blocks=nb)
    src = OracleSeq(num_tokens=0)
    opm.allocate(src, num_tokens + 9)
    dsts = [OracleSeq(num_tokens=0) for _ in range(n)]
    assert ok.cpu().bool().tolist() == opm.fork(src, dsts, num_tokens)
    tables, lens, free, top, rc = to_dense(opm, [src] + dsts, 8)
    assert np.array_equal(pm.tables.cpu().numpy(), tables)
    assert np.array_equal(pm.lens.cpu().numpy(), lens)
    assert int(pm.free_top.item()) == int(top)
    assert np.array_equal(pm.free_list[:int(top)].cpu().numpy(), free[:int(top)])
    assert np.array_equal(pm.ref_counts_dev.cpu().numpy(), rc)
    # the partial page's rows were copied into every branch's own block
    full, part = divmod(num_tokens, bs)
    if part:
        sb = int(pm.tables[0, full])
        for i in range(n):
            db = int(pm.tables[1 + i, full])
            assert db != sb
            assert torch.equal(cache.pages[:, :, db, :part], cache.pages[:, :, sb, :part])
    # releasing the branches gives back exactly their private blocks
    pm.free_rows(1, n)
    torch.cuda.synchronize()
    assert pm.lens[1:].sum().item() == 0
    assert int(pm.free_top.item()) == nb - int(pm.lens[0].item())


@pytest.mark.parametrize("preset", ["toy-draft", "tp-draft"])
def test_draft_branches_equal_one_by_one(cuda, preset):
    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.models.gemma_adapter import GemmaAdapter

    dt = torch.float32 if preset.startswith("toy") else torch.bfloat16
    w = GemmaWeights.random(PRESETS[preset], seed=77, dtype=dt, device=cuda, max_pos=512)
    rng = np.random.default_rng(5)
    prefix = [int(x) for x in rng.integers(0, w.shape.vocab, 45)]
    feeds = [[int(x) for x in rng.integers(0, w.shape.vocab, a + 1)] for a in (0, 1, 4, 2, 0, 3, 1)]
    k = 4
    a = GemmaAdapter(w, max_model_len=256, name="draft", max_branches=10)
    got = a.draft_branches(prefix, feeds, k)
    ref_adapter = GemmaAdapter(w, max_model_len=256, name="draft")
    want = [ref_adapter.draft_speculate(prefix + f, k)[0] for f in feeds]
    assert got == want
    # the trunk row and the page pool are intact afterwards: the next call reuses the prefix
    assert a.cached == prefix
    assert a.draft_branches(prefix, feeds[:2], k) == want[:2]
