"""CPU: pin the oracle to the reference's golden vectors and check its internal consistency."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import page_manager as opm
from oracle import spec_cache as osc
from oracle.engine import greedy_sd
from oracle.gemma import GemmaShape, OracleGemma, bf16_round, greedy_ar, init_weights, new_pages
from oracle.paged_kv import attention_ref, paged_verify_attention, verify_mask, write_kv
from oracle.verify import verify_greedy, verify_sample


def _greedy_cases():
    z = np.load(GOLDEN / "verify_greedy.npz")
    names = sorted({k.split("__")[0] for k in z.files})
    return [(n, z[f"{n}__logits"], z[f"{n}__spec"], z[f"{n}__accept_until"], z[f"{n}__recovery"]) for n in names]


@pytest.mark.parametrize("case", _greedy_cases(), ids=lambda c: c[0])
def test_oracle_greedy_matches_reference_goldens(case):
    _, lp, spec, acc_ref, rec_ref = case
    acc, rec, mask = verify_greedy(lp, spec)
    np.testing.assert_array_equal(acc, acc_ref)
    np.testing.assert_array_equal(rec, rec_ref)
    k = spec.shape[1] - 1
    assert not mask[:, 0].any()
    np.testing.assert_array_equal(mask[:, 1:], np.arange(k)[None] < acc[:, None])


def _replay(scn):
    pm = opm.OraclePageManager(scn["block_size"], scn["num_blocks"])
    seqs = [opm.OracleSeq(num_tokens=n) for n in scn["prompts"]]
    for op in scn["ops"]:
        s = seqs[op["seq"]] if "seq" in op else None
        if op["op"] == "allocate":
            assert pm.allocate(s, op["num_tokens"]) == op["ret"]
        elif op["op"] == "allocate_draft":
            assert pm.allocate_draft(s, op["num_tokens"]) == op["ret"]
        elif op["op"] == "append":
            s.num_tokens += op["n"]
        elif op["op"] == "rollback":
            pm.rollback_speculative(s, op["accepted"], op["reserved"])
        elif op["op"] == "free":
            pm.free_sequence(s)
        elif op["op"] == "share":
            src, dst = seqs[op["src"]], seqs[op["dst"]]
            dst.block_table.extend(src.block_table)
            for b in src.block_table:
                pm.ref_counts[b] += 1
        after = op["after"]
        assert pm.free_blocks == after["free_blocks"], op
        assert {str(k): v for k, v in sorted(pm.ref_counts.items())} == after["ref_counts"], op
        assert [q.block_table for q in seqs] == after["block_tables"], op
        assert [q.draft_block_table for q in seqs] == after["draft_block_tables"], op
    return pm, seqs


def test_oracle_page_manager_matches_reference_traces():
    scenarios = json.loads((GOLDEN / "page_manager.json").read_text())
    assert len(scenarios) >= 8
    for scn in scenarios:
        _replay(scn)
    # the reference's tests/test_page_rollback.py scenario, as its page manager answered it
    first = scenarios[0]["ops"]
    assert first[0]["after"]["block_tables"] == [[9, 8, 7, 6]]
    assert first[1]["after"]["block_tables"] == [[9, 8]]
    assert first[1]["after"]["free_blocks"] == list(range(8))


def test_dense_rollback_equals_list_semantics():
    rng = np.random.default_rng(5)
    for trial in range(20):
        bs = int(rng.choice([4, 16]))
        nb = 64
        pm = opm.OraclePageManager(bs, nb)
        seqs = [opm.OracleSeq(num_tokens=int(rng.integers(1, 30))) for _ in range(5)]
        for q in seqs:
            pm.allocate(q, int(rng.integers(1, 40)))
        # share a few blocks to exercise ref counts > 1
        for blk in seqs[0].block_table[:2]:
            seqs[1].block_table.append(blk)
            pm.ref_counts[blk] += 1
        tables, lens, free, top, rc = opm.to_dense(pm, seqs, max_blocks=32)
        ntok = np.array([q.num_tokens for q in seqs], np.int32)
        acc = rng.integers(0, 6, len(seqs)).astype(np.int32)
        for q, a in zip(seqs, acc):
            pm.rollback_speculative(q, int(a), 0)
        t2, l2, f2, top2, rc2 = opm.dense_rollback(tables, lens, free, top, rc, ntok, acc, bs)
        e = opm.to_dense(pm, seqs, max_blocks=32)
        np.testing.assert_array_equal(t2, e[0])
        np.testing.assert_array_equal(l2, e[1])
        np.testing.assert_array_equal(f2[:top2], e[2][: e[3]])
        assert top2 == e[3]
        np.testing.assert_array_equal(rc2, e[4])


def test_dense_allocate_equals_list_semantics():
    rng = np.random.default_rng(9)
    for trial in range(20):
        pm = opm.OraclePageManager(16, 20)
        seqs = [opm.OracleSeq(num_tokens=int(rng.integers(0, 40))) for _ in range(6)]
        tables, lens, free, top, rc = opm.to_dense(pm, seqs, max_blocks=16)
        n_new = rng.integers(0, 60, len(seqs)).astype(np.int32)
        ok_list = [pm.allocate(q, int(n)) for q, n in zip(seqs, n_new)]
        ntok = np.array([q.num_tokens for q in seqs], np.int32)
        t2, l2, f2, top2, rc2, ok = opm.dense_allocate(tables, lens, free, top, rc, ntok, n_new, 16)
        e = opm.to_dense(pm, seqs, max_blocks=16)
        np.testing.assert_array_equal(ok, ok_list)
        np.testing.assert_array_equal(t2, e[0])
        assert top2 == e[3]
        np.testing.assert_array_equal(rc2, e[4])


def test_oracle_spec_cache_known_answers():
    cases = json.loads((GOLDEN / "spec_cache.json").read_text())
    c = cases["ref_hit_and_miss"]
    n, k, v = c["num_branches"], c["k"], c["vocab"]
    keys = np.zeros((n, 3), np.int32)
    toks = np.zeros((n, k), np.int32)
    lg = np.zeros((n, k, v), np.float32)
    valid = np.zeros(n, bool)
    for ins in c["inserts"]:
        keys[ins["slot"]] = ins["key"]
        toks[ins["slot"]] = ins["tokens"]
        valid[ins["slot"]] = True
    for lk in c["lookups"]:
        hit, idx, tok, _ = osc.lookup(keys, toks, lg, valid, np.array([lk["key"]], np.int32))
        assert bool(hit[0]) == lk["hit"]
        assert int(idx[0]) == lk["idx"]
        assert tok[0].tolist() == lk["tokens"]


def test_oracle_sample_properties():
    rng = np.random.default_rng(3)
    b, k, v = 4, 4, 50
    lp = rng.standard_normal((b, k + 1, v)).astype(np.float32)
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    ua = rng.random((b, k), dtype=np.float32)
    ug = rng.random((b, v), dtype=np.float32) * 0.999 + 0.0005
    # draft == target distribution at the judged rows -> every ratio is 1 -> all accepted
    lq = lp[:, 1:, :].copy()
    acc, rec, mask = verify_sample(lp, lq, spec, ua, ug, alignment="reference")
    assert (acc == k).all()
    # u = 1 - eps never accepts unless ratio == 1; u = 0 always accepts
    lq2 = rng.standard_normal((b, k, v)).astype(np.float32)
    acc0, _, _ = verify_sample(lp, lq2, spec, np.zeros((b, k), np.float32), ug)
    assert (acc0 == k).all()
    # residual draw never returns a token with zero residual mass (x = 1, p == q)
    acc1, rec1, _ = verify_sample(lp, lp[:, :k], spec, np.full((b, k), 0.999999, np.float32), ug,
                                  sampler_x=1.0, alignment="standard")
    assert (acc1 == k).all()  # ratio 1 everywhere under standard alignment


def test_verify_mask_and_attention():
    m = verify_mask(3, 2)
    assert m.shape == (2, 5)
    assert np.isinf(m[0, 4]) and m[1, 4] == 0 and m[0, 3] == 0
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 8))
    kk = rng.standard_normal((5, 8))
    vv = rng.standard_normal((5, 8))
    o = attention_ref(q, kk, vv, m)
    assert np.isfinite(o).all()


def test_paged_attention_oracle_matches_dense():
    rng = np.random.default_rng(1)
    hq, hkv, d, bs, nb = 4, 2, 16, 4, 12
    pages = np.zeros((2, 1, nb, bs, hkv, d), np.float32)
    table = rng.permutation(nb).astype(np.int32)[None, :]
    n = 13
    k = rng.standard_normal((1, n, hkv, d)).astype(np.float32)
    v = rng.standard_normal((1, n, hkv, d)).astype(np.float32)
    write_kv(pages, 0, table, np.arange(n)[None], k, v)
    q = rng.standard_normal((1, 3, hq, d)).astype(np.float32)
    out = paged_verify_attention(q, pages, 0, table, np.array([n]))
    for h in range(hq):
        ref = attention_ref(q[0, :, h], k[0, :, h // 2], v[0, :, h // 2], verify_mask(n - 3, 3))
        np.testing.assert_allclose(out[0, :, h], ref, rtol=1e-12, atol=1e-12)


def test_bf16_round():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3333, 65504.0], np.float32)
    r = bf16_round(x)
    import torch

    np.testing.assert_array_equal(r, torch.tensor(x).bfloat16().float().numpy())


TOY_T = GemmaShape(2, 256, 4, 1, 64, 1024, 1024)
TOY_D = GemmaShape(1, 256, 4, 1, 64, 1024, 1024)


def test_oracle_sd_stream_equals_ar_stream_toy():
    t = OracleGemma(TOY_T, init_weights(TOY_T, 0))
    d = OracleGemma(TOY_D, init_weights(TOY_D, 1))
    for seed in range(3):
        p = np.random.default_rng(seed).integers(0, 1024, 64)
        ar = greedy_ar(t, p, 24)
        sd, _ = greedy_sd(t, d, p, 24)
        assert sd == ar
        sd2, steps = greedy_sd(t, t, p, 24)  # self-speculation: every draft accepted
        assert sd2 == ar and steps <= 24 // 5 + 1


def test_oracle_gemma_matches_transformers_fp32():
    """Cross-check the restated Gemma math against transformers' torch GemmaForCausalLM (fp32)."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    from transformers import GemmaConfig, GemmaForCausalLM

    shape = GemmaShape(2, 64, 4, 2, 16, 128, 97)
    w = init_weights(shape, 7)
    cfg = GemmaConfig(vocab_size=shape.vocab, hidden_size=shape.d_model, intermediate_size=shape.ffn,
                      num_hidden_layers=shape.num_layers, num_attention_heads=shape.num_heads,
                      num_key_value_heads=shape.num_kv_heads, head_dim=shape.head_dim,
                      hidden_activation="gelu_pytorch_tanh", rms_norm_eps=shape.eps, rope_theta=shape.rope_theta,
                      max_position_embeddings=256, tie_word_embeddings=True, attention_bias=False)
    cfg._attn_implementation = "eager"
    m = GemmaForCausalLM(cfg).float().eval()
    sd = m.state_dict()
    t = lambda a: torch.tensor(a)  # noqa: E731
    sd["model.embed_tokens.weight"] = t(w["embed"])
    sd["model.norm.weight"] = t(w["final_norm"])
    for i, lw in enumerate(w["layers"]):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = t(lw["attn_norm"])
        sd[p + "post_attention_layernorm.weight"] = t(lw["mlp_norm"])
        sd[p + "self_attn.q_proj.weight"] = t(lw["wq"])
        sd[p + "self_attn.k_proj.weight"] = t(lw["wk"])
        sd[p + "self_attn.v_proj.weight"] = t(lw["wv"])
        sd[p + "self_attn.o_proj.weight"] = t(lw["wo"])
        sd[p + "mlp.gate_proj.weight"] = t(lw["wg"])
        sd[p + "mlp.up_proj.weight"] = t(lw["wu"])
        sd[p + "mlp.down_proj.weight"] = t(lw["wd"])
    if "lm_head.weight" in sd:
        sd["lm_head.weight"] = t(w["embed"])
    m.load_state_dict(sd)
    ids = np.random.default_rng(0).integers(0, shape.vocab, 11)
    with torch.no_grad():
        ref = m(torch.tensor(ids)[None]).logits[0].numpy()
    om = OracleGemma(shape, w, "fp32", max_pos=256)
    pages = new_pages(shape, 4, 4)
    table = np.arange(4, dtype=np.int32)[None]
    # prompt split in two calls exercises the paged cache
    a = om.forward(ids[None, :7], pages, table, [0])
    b = om.forward(ids[None, 7:], pages, table, [7])
    got = np.concatenate([a[0], b[0]], 0)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_oracle_folded_norm_formulation_matches_textbook_fp32():
    """Folding the RMSNorm weights into q/k/v and gate/up is exact math: fp32 results agree to rounding."""
    from oracle.gemma import fold_norms

    w = init_weights(TOY_T, 4)
    a = OracleGemma(TOY_T, w, "fp32")
    b = OracleGemma(TOY_T, fold_norms(w), "fp32")
    assert b.folded and not a.folded
    ids = np.random.default_rng(1).integers(0, TOY_T.vocab, (1, 21))
    pa, pb = new_pages(TOY_T, 4, 16), new_pages(TOY_T, 4, 16)
    table = np.arange(4, dtype=np.int32)[None]
    la = a.forward(ids, pa, table, [0])
    lb = b.forward(ids, pb, table, [0])
    np.testing.assert_allclose(la, lb, rtol=1e-4, atol=1e-5)


def test_oracle_fork_shares_and_frees():
    """Branch fork: full trunk blocks shared (ref counts), a private block per branch for the
    partial page; freeing every row returns all blocks to the free list."""
    from oracle.page_manager import OraclePageManager, OracleSeq

    pm = OraclePageManager(block_size=16, num_blocks=32)
    src = OracleSeq(num_tokens=40)
    assert pm.allocate(src, 0) and len(src.block_table) == 3
    dsts = [OracleSeq(num_tokens=40) for _ in range(3)]
    assert pm.fork(src, dsts, 40) == [True, True, True]
    for d in dsts:
        assert d.block_table[:2] == src.block_table[:2] and d.block_table[2] not in src.block_table
    assert pm.ref_counts[src.block_table[0]] == 4 and pm.ref_counts[src.block_table[2]] == 1
    for q in dsts + [src]:
        pm.free_sequence(q)
    assert sorted(pm.free_blocks) == list(range(32)) and pm.ref_counts == {}
    # page-aligned trunk: nothing popped
    pm2 = OraclePageManager(block_size=16, num_blocks=8)
    s2 = OracleSeq(num_tokens=32)
    pm2.allocate(s2, 0)
    top = len(pm2.free_blocks)
    d2 = OracleSeq(num_tokens=32)
    assert pm2.fork(s2, [d2], 32) == [True] and len(pm2.free_blocks) == top and d2.block_table == s2.block_table


def test_top_p_threshold_definition():
    """Nucleus cutoff of softmax(x / T): the value at which the running mass (descending, fp64) first
    reaches p * Z; ties at the cutoff stay, NaN and -inf go."""
    from oracle.verify import top_p_mask, top_p_threshold

    x = np.array([2, 1, 1, 0], np.float32)  # masses 1, e^-1, e^-1, e^-2 (Z = 1.871)
    assert top_p_threshold(x, 1.0, 0.5) == 2.0       # 1 >= 0.936
    assert top_p_threshold(x, 1.0, 0.6) == 1.0       # 1 < 1.123 <= 1.368: both tied 1s kept
    assert top_p_threshold(x, 1.0, 0.99) == 0.0
    assert top_p_threshold(x, 1.0, 1e-9) == 2.0
    assert top_p_threshold(x, 0.25, 0.9) == 2.0      # sharper: e^-4 tails
    got = top_p_mask(np.array([[2, 1, 1, 0, np.nan, -np.inf]], np.float32), 1.0, 0.6)
    np.testing.assert_array_equal(got, [[2, 1, 1, -np.inf, -np.inf, -np.inf]])
    assert top_p_threshold(np.array([np.nan, -np.inf], np.float32), 1.0, 0.9) is None
    np.testing.assert_array_equal(top_p_mask(x[None], 1.0, 1.0), x[None])  # p >= 1: untouched
