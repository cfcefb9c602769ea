"""Host-side pieces of the reference's public surface (no GPU): dense masks, the
KV gather helper on a CPU cache, worker and loader defaults."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.paged_kv import branch_mask, slot_of, verify_mask


@pytest.mark.parametrize("seq_len,query_len", [(0, 1), (7, 5), (33, 1), (16, 16)])
def test_verify_mask_equals_reference(seq_len, query_len):
    from ssd_b200.kernels.masks import build_verify_mask

    got = build_verify_mask(seq_len, query_len, device="cpu").numpy()
    np.testing.assert_array_equal(got, verify_mask(seq_len, query_len))


@pytest.mark.parametrize("b,nb,trunk,branch", [(1, 3, 4, 2), (2, 2, 0, 3), (1, 1, 5, 0)])
def test_branch_mask_equals_reference(b, nb, trunk, branch):
    from ssd_b200.kernels.masks import build_branch_mask

    got = build_branch_mask(b, nb, trunk, branch, device="cpu").numpy()
    np.testing.assert_array_equal(got, branch_mask(b, nb, trunk, branch))


def test_gather_kv_for_positions_reads_the_slots():
    from ssd_b200.kernels.kv_cache import KVCacheState, gather_kv_for_positions

    cache = KVCacheState.allocate(2, 6, 4, 2, 8, dtype=torch.float32, device="cpu")
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=torch.Generator().manual_seed(0)))
    table = np.array([5, 2, 0], dtype=np.int32)
    pos = np.array([0, 3, 4, 9, 11], dtype=np.int64)
    k, v = gather_kv_for_positions(cache, 1, table, pos)
    slots = slot_of(table, pos, 4)
    flat = cache.pages.reshape(2, 2, 6 * 4, 2, 8)
    np.testing.assert_array_equal(k.numpy(), flat[0, 1, slots].numpy())
    np.testing.assert_array_equal(v.numpy(), flat[1, 1, slots].numpy())


def test_worker_and_loader_defaults(monkeypatch):
    from ssd_b200.models.model_loader import default_draft_path, default_target_path
    from ssd_b200.runtime.workers import WorkerConfig

    wc = WorkerConfig()
    assert wc.use_toy is True and wc.instance_mode is False
    monkeypatch.delenv("TARGET_MODEL_PATH", raising=False)
    monkeypatch.setenv("DRAFT_MODEL_PATH", "toy-draft")
    assert default_target_path() == "gemma-7b"
    assert default_draft_path() == "toy-draft"


def test_gemma_adapter_takes_the_reference_arguments():
    import inspect

    from ssd_b200.models.gemma_adapter import GemmaAdapter

    params = list(inspect.signature(GemmaAdapter.__init__).parameters.values())[1:]
    # the reference's positional order (gemma_adapter.py:28-36) ...
    names = ["model_path", "vocab_size", "share_key", "mesh", "devices", "role"]
    assert [q.name for q in params[:6]] == names
    assert all(q.kind is inspect.Parameter.POSITIONAL_OR_KEYWORD for q in params[:6])
    # ... and everything the adapter adds is keyword-only, so GemmaAdapter(path, 256000) cannot
    # set a cache size by position
    assert all(q.kind is inspect.Parameter.KEYWORD_ONLY for q in params[6:])
