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


@pytest.mark.parametrize("preset", ["toy-draft", "tp-draft"])
def test_draft_speculate_chained_equals_token_by_token(cuda, preset):
    """``draft_speculate`` (draft tokens chained on the device, one upload and one download per
    call) gives the tokens, logits, cache contents and page tables of the token-by-token loop
    (truncate, then one forward and one host-side argmax per token) over a sequence of calls that
    extend the prefix, roll it back, and ask for the bonus row."""
    from ssd_b200.algorithm.verify import argmax_rows
    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.models.gemma_adapter import GemmaAdapter

    dt = torch.float32 if preset.startswith("toy") else torch.bfloat16
    w = GemmaWeights.random(PRESETS[preset], seed=78, dtype=dt, device=cuda, max_pos=512)
    fast = GemmaAdapter(w, max_model_len=256, name="draft")
    slow = GemmaAdapter(w, max_model_len=256, name="draft")

    def token_by_token(a, prefix, k, with_bonus):
        common = 0
        for x, y in zip(a.cached, prefix):
            if x != y:
                break
            common += 1
        common = min(common, len(prefix) - 1)
        a._truncate(common)
        rows = k + 1 if with_bonus else k
        logits = torch.empty((rows, a.vocab_size), dtype=torch.float32, device=cuda)
        feed, spec = prefix[common:], []
        nxt = torch.empty(1, dtype=torch.int32, device=cuda)
        for i in range(rows):
            lg = a._run(feed, a._lg1, last_only=True)
            logits[i].copy_(lg[0])
            if i == k:
                break
            argmax_rows(lg, nxt)
            spec.append(int(nxt.item()))
            feed = [spec[-1]]
        return spec, logits

    rng = np.random.default_rng(9)
    prefix = [int(x) for x in rng.integers(0, w.shape.vocab, 70)]
    calls = []
    for step in range(6):
        k = 4 if step != 3 else 0
        calls.append((list(prefix), k, step % 2 == 0 or k == 0))
        prefix = prefix + [int(x) for x in rng.integers(0, w.shape.vocab, 1 + step % 2)]
        if step == 4:
            prefix = prefix[:60] + [int(x) for x in rng.integers(0, w.shape.vocab, 3)]  # a rollback
    for prefix, k, bonus in calls:
        got, lg_got = fast.draft_speculate(prefix, k, with_bonus=bonus)
        want, lg_want = token_by_token(slow, prefix, k, bonus)
        assert got == want
        assert torch.equal(lg_got, lg_want)
        assert fast.cached == slow.cached
        torch.cuda.synchronize()
        assert torch.equal(fast.pm.tables, slow.pm.tables) and torch.equal(fast.pm.lens, slow.pm.lens)
