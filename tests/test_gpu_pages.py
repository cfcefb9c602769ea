"""GPU parity: page allocation / rollback / free kernels (K5) vs the reference's traces (bit-exact)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import page_manager as opm

pytestmark = pytest.mark.gpu


def test_device_page_manager_replays_reference_traces(cuda):
    import torch

    from ssd_b200.runtime.page_manager import PageManager
    from ssd_b200.runtime.sequence import Sequence

    scenarios = json.loads((GOLDEN / "page_manager.json").read_text())
    for scn in scenarios:
        pm = PageManager(scn["block_size"], scn["num_blocks"], max_seqs=8)
        seqs = [Sequence(seq_id=i, prompt_token_ids=list(range(n))) for i, n in enumerate(scn["prompts"])]
        for op in scn["ops"]:
            s = seqs[op["seq"]] if "seq" in op else None
            if op["op"] == "allocate":
                assert pm.allocate(s, op["num_tokens"]) == op["ret"]
            elif op["op"] == "allocate_draft":
                assert pm.allocate_draft(s, op["num_tokens"]) == op["ret"]
            elif op["op"] == "append":
                s.append_tokens(list(range(op["n"])))
            elif op["op"] == "rollback":
                pm.rollback_speculative(s, op["accepted"], op["reserved"])
            elif op["op"] == "free":
                pm.free_sequence(s)
            elif op["op"] == "share":
                src, dst = seqs[op["src"]], seqs[op["dst"]]
                rs, rd = pm.row(src), pm.row(dst)
                n = len(src.block_table)
                pm.tables[rd, :n] = pm.tables[rs, :n]
                pm.lens[rd] = n
                for blk in src.block_table:
                    pm.ref_counts_dev[blk] += 1
                dst.block_table[:] = list(src.block_table)
            after = op["after"]
            assert pm.free_blocks == after["free_blocks"], (scn["name"], op)
            assert {str(k): v for k, v in sorted(pm.ref_counts.items())} == after["ref_counts"], (scn["name"], op)
            assert [q.block_table for q in seqs] == after["block_tables"], (scn["name"], op)
            assert [q.draft_block_table for q in seqs] == after["draft_block_tables"], (scn["name"], op)
        torch.cuda.synchronize()


def _dev_state(tables, lens, free, top, rc):
    import torch

    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.int32, device="cuda")  # noqa: E731
    return t(tables), t(lens), t(free), t([int(top)]), t(rc)


@pytest.mark.parametrize("nseq", [1, 7, 300, 1500])
def test_batched_rollback_bit_exact(cuda, nseq):
    import torch

    from ssd_b200 import _lib

    rng = np.random.default_rng(nseq)
    bs, nb, mb = 4, 8 * nseq + 64, 24
    pm = opm.OraclePageManager(bs, nb)
    seqs = [opm.OracleSeq(num_tokens=int(rng.integers(1, 30))) for _ in range(nseq)]
    for q in seqs:
        pm.allocate(q, int(rng.integers(1, 50)))
    for i in range(0, nseq - 1, 3):  # shared blocks: ref counts 2 and 3
        for blk in seqs[i].block_table[:2]:
            if len(seqs[i + 1].block_table) < mb:
                seqs[i + 1].block_table.append(blk)
                pm.ref_counts[blk] += 1
    st = opm.to_dense(pm, seqs, mb)
    ntok = np.array([q.num_tokens for q in seqs], np.int32)
    acc = rng.integers(0, 6, nseq).astype(np.int32)
    exp = opm.dense_rollback(*st, ntok, acc, bs)
    tb, ln, fr, top, rc = _dev_state(*st)
    nt, ac = torch.tensor(ntok, device="cuda"), torch.tensor(acc, device="cuda")
    kv = torch.zeros(nseq, dtype=torch.int32, device="cuda")
    so = _lib.lib()
    rc_ = so.ssd_page_rollback(_lib.stream_ptr(), tb.data_ptr(), ln.data_ptr(), mb, fr.data_ptr(), top.data_ptr(),
                               rc.data_ptr(), nb, nt.data_ptr(), ac.data_ptr(), kv.data_ptr(), bs, nseq)
    assert rc_ == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tb.cpu().numpy(), exp[0])
    np.testing.assert_array_equal(ln.cpu().numpy(), exp[1])
    t2 = int(top.item())
    assert t2 == int(exp[3])
    np.testing.assert_array_equal(fr.cpu().numpy()[:t2], exp[2][:t2])
    np.testing.assert_array_equal(rc.cpu().numpy(), exp[4])
    np.testing.assert_array_equal(kv.cpu().numpy(), ntok + acc)


@pytest.mark.parametrize("nseq", [5, 1100])
def test_batched_allocate_bit_exact(cuda, nseq):
    import torch

    from ssd_b200 import _lib

    rng = np.random.default_rng(nseq + 1)
    bs, nb, mb = 16, 6 * nseq, 12
    pm = opm.OraclePageManager(bs, nb)
    seqs = [opm.OracleSeq(num_tokens=int(rng.integers(0, 40))) for _ in range(nseq)]
    st = opm.to_dense(pm, seqs, mb)
    ntok = np.array([q.num_tokens for q in seqs], np.int32)
    n_new = rng.integers(0, 150, nseq).astype(np.int32)  # some requests exceed the pool / table
    exp = opm.dense_allocate(*st, ntok, n_new, bs)
    tb, ln, fr, top, rc = _dev_state(*st)
    ok = torch.zeros(nseq, dtype=torch.uint8, device="cuda")
    nt, nn = torch.tensor(ntok, device="cuda"), torch.tensor(n_new, device="cuda")
    so = _lib.lib()
    assert so.ssd_page_allocate(_lib.stream_ptr(), tb.data_ptr(), ln.data_ptr(), mb, fr.data_ptr(), top.data_ptr(),
                                rc.data_ptr(), nb, nt.data_ptr(), nn.data_ptr(), ok.data_ptr(), bs, nseq) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ok.cpu().numpy().astype(bool), exp[5])
    np.testing.assert_array_equal(tb.cpu().numpy(), exp[0])
    np.testing.assert_array_equal(ln.cpu().numpy(), exp[1])
    assert int(top.item()) == int(exp[3])
    np.testing.assert_array_equal(rc.cpu().numpy(), exp[4])


def test_reference_api_reuses_freed_slots(cuda):
    # More sequences than device slots through allocate / free_sequence (page_manager.py:21-64): a freed
    # sequence gives its slot back, and a full manager says so instead of failing inside a generator.
    from ssd_b200.runtime.page_manager import PageManager
    from ssd_b200.runtime.sequence import Sequence

    pm = PageManager(16, 64, max_seqs=4)
    for i in range(3 * pm.max_seqs):
        s = Sequence(seq_id=i, prompt_token_ids=list(range(20)))
        assert pm.allocate(s, 5)
        assert len(s.block_table) == 2
        pm.free_sequence(s)
        assert s.block_table == [] and sorted(pm.free_blocks) == list(range(64)) and pm.ref_counts == {}
    held = [Sequence(seq_id=100 + i, prompt_token_ids=[1, 2, 3]) for i in range(pm.max_seqs)]
    for s in held:
        assert pm.allocate(s, 1)
    with pytest.raises(RuntimeError, match="slots"):
        pm.allocate(Sequence(seq_id=999, prompt_token_ids=[1]), 1)
