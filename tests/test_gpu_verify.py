"""GPU parity: fused acceptance kernels (K4) vs the oracle and the reference's goldens."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN
from oracle.verify import verify_greedy as o_greedy
from oracle.verify import verify_sample as o_sample

pytestmark = pytest.mark.gpu


def _greedy_cases():
    z = np.load(GOLDEN / "verify_greedy.npz")
    names = sorted({k.split("__")[0] for k in z.files})
    return [(n, z[f"{n}__logits"], z[f"{n}__spec"], z[f"{n}__accept_until"], z[f"{n}__recovery"]) for n in names]


@pytest.mark.parametrize("case", _greedy_cases(), ids=lambda c: c[0])
def test_greedy_matches_reference_goldens(cuda, case):
    from ssd_b200.algorithm.verify import verify_greedy

    _, lp, spec, acc_ref, rec_ref = case
    res = verify_greedy(lp, spec)
    np.testing.assert_array_equal(res.accept_until.cpu().numpy(), acc_ref)
    np.testing.assert_array_equal(res.recovery_tokens.cpu().numpy(), rec_ref)
    _, _, mask = o_greedy(lp, spec)
    np.testing.assert_array_equal(res.accepted_mask.cpu().numpy(), mask)


@pytest.mark.parametrize("b,k,v", [(8, 4, 256000), (32, 6, 32000), (3, 1, 4099), (1, 8, 7), (3, 63, 515)])
def test_greedy_bit_exact_vs_oracle(cuda, b, k, v):
    from ssd_b200.algorithm.verify import verify_greedy

    rng = np.random.default_rng(b * 1000 + v)
    lp = (3.0 * rng.standard_normal((b, k + 1, v))).astype(np.float32)
    t = lp.argmax(-1)
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    for i in range(b):  # ladder of accept lengths
        a = i % (k + 1)
        spec[i, 1:a + 1] = t[i, :a]
    # plant exact ties at a later index: first index must still win
    lp[0, 0, v - 1] = lp[0, 0].max()
    res, tt = verify_greedy(lp, spec, target_tokens=True)
    acc, rec, mask = o_greedy(lp, spec)
    np.testing.assert_array_equal(res.accept_until.cpu().numpy(), acc)
    np.testing.assert_array_equal(res.recovery_tokens.cpu().numpy(), rec)
    np.testing.assert_array_equal(res.accepted_mask.cpu().numpy(), mask)
    np.testing.assert_array_equal(tt.cpu().numpy(), lp.argmax(-1))


def test_greedy_repeat_calls_reuse_workspace(cuda):
    from ssd_b200.algorithm.verify import verify_greedy

    rng = np.random.default_rng(0)
    for _ in range(5):
        lp = rng.standard_normal((4, 5, 50000)).astype(np.float32)
        spec = rng.integers(0, 50000, (4, 5)).astype(np.int32)
        res = verify_greedy(lp, spec)
        acc, rec, _ = o_greedy(lp, spec)
        np.testing.assert_array_equal(res.recovery_tokens.cpu().numpy(), rec)


def test_argmax_rows(cuda):
    import torch

    from ssd_b200.algorithm.verify import argmax_rows

    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 256000)).astype(np.float32)
    x[3, 100] = x[3, 200] = 50.0
    got = argmax_rows(torch.tensor(x, device="cuda")).cpu().numpy()
    np.testing.assert_array_equal(got, x.argmax(-1))
    assert got[3] == 100


def _sample_inputs(b, k, v, seed, scale=3.0):
    rng = np.random.default_rng(seed)
    lp = (scale * rng.standard_normal((b, k + 1, v))).astype(np.float32)
    lq = (scale * rng.standard_normal((b, k, v))).astype(np.float32)
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    # make draft tokens plausible under both models so that some are accepted
    for i in range(b):
        for j in range(k):
            tok = int(lq[i, j].argmax())
            spec[i, j + 1] = tok
            lp[i, j + 1, tok] = lq[i, j, tok] + rng.normal(0.0, 0.5)
            lp[i, j, tok] = lq[i, j, tok] + rng.normal(0.0, 0.5)
    ua = rng.random((b, k), dtype=np.float32)
    ug = np.clip(rng.random((b, v), dtype=np.float32), 1e-7, 1 - 1e-7).astype(np.float32)
    return lp, lq, spec, ua, ug


@pytest.mark.parametrize("alignment", ["reference", "standard"])
@pytest.mark.parametrize("b,k,v,tp,tq", [(8, 4, 256000, 1.0, 1.0), (6, 3, 4099, 0.7, 1.3), (16, 6, 1024, 1.0, 0.5),
                                          (2, 63, 300, 1.0, 1.0)])
def test_sample_matches_oracle(cuda, alignment, b, k, v, tp, tq):
    from ssd_b200.algorithm.verify import verify_sample

    lp, lq, spec, ua, ug = _sample_inputs(b, k, v, seed=b + k + v)
    res = verify_sample(lp, lq, spec, (ua, ug), temperature_p=tp, temperature_q=tq, sampler_x=0.5,
                        alignment=alignment)
    acc, rec, mask, (am, gap) = o_sample(lp, lq, spec, ua, ug, temperature_p=tp, temperature_q=tq,
                                         sampler_x=0.5, alignment=alignment, return_margins=True)
    ga = res.accept_until.cpu().numpy()
    gr = res.recovery_tokens.cpu().numpy()
    # Bit-exact except near-ties: |u - ratio| or the Gumbel top-2 gap within fp32
    # exp/log rounding noise (the CUDA and numpy exp/log differ by a few ulp).
    near_acc = am < 1e-5
    assert np.all((ga == acc) | near_acc), (ga, acc, am)
    ok_rows = ga == acc
    near_gap = gap < 1e-4
    assert np.all((gr == rec) | near_gap | ~ok_rows), (gr, rec, gap)
    exact = ok_rows & ~near_gap
    assert exact.sum() >= len(exact) - 1
    assert 0 < acc.sum()  # some acceptance happened
    np.testing.assert_array_equal(res.accepted_mask.cpu().numpy()[ok_rows], mask[ok_rows])


def test_sample_bonus_and_full_accept(cuda):
    from ssd_b200.algorithm.verify import verify_sample

    b, k, v = 4, 4, 3000
    rng = np.random.default_rng(11)
    lp = rng.standard_normal((b, k + 1, v)).astype(np.float32)
    lq = lp[:, 1:, :].copy()   # reference alignment: ratio == 1 everywhere -> bonus draw from lp[k]
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    ua = rng.random((b, k), dtype=np.float32) * 0.99
    ug = np.clip(rng.random((b, v), dtype=np.float32), 1e-7, 1 - 1e-7).astype(np.float32)
    res = verify_sample(lp, lq, spec, (ua, ug))
    acc, rec, _, (_, gap) = o_sample(lp, lq, spec, ua, ug, return_margins=True)
    assert (res.accept_until.cpu().numpy() == k).all() and (acc == k).all()
    gr = res.recovery_tokens.cpu().numpy()
    assert np.all((gr == rec) | (gap < 1e-4))


@pytest.mark.parametrize("alignment", ["reference", "standard"])
def test_sample_k0_draws_the_bonus_token(cuda, alignment):
    # verify.py:98-114 with k = 0: nothing to accept, the bonus token comes from softmax(lp[0] / Tp)
    from ssd_b200.algorithm.verify import verify_sample

    b, v = 5, 4099
    rng = np.random.default_rng(21)
    lp = (3.0 * rng.standard_normal((b, 1, v))).astype(np.float32)
    lq = np.zeros((b, 0, v), np.float32)
    spec = rng.integers(0, v, (b, 1)).astype(np.int32)
    ua = np.zeros((b, 0), np.float32)
    ug = np.clip(rng.random((b, v), dtype=np.float32), 1e-7, 1 - 1e-7).astype(np.float32)
    res = verify_sample(lp, lq, spec, (ua, ug), temperature_p=0.8, alignment=alignment)
    acc, rec, mask, (_, gap) = o_sample(lp, lq, spec, ua, ug, temperature_p=0.8, alignment=alignment,
                                        return_margins=True)
    assert (acc == 0).all() and (res.accept_until.cpu().numpy() == 0).all()
    gr = res.recovery_tokens.cpu().numpy()
    assert np.all((gr == rec) | (gap < 1e-4)), (gr, rec, gap)
    assert ((gr == rec) & (gap >= 1e-4)).sum() >= b - 1
    np.testing.assert_array_equal(res.accepted_mask.cpu().numpy(), mask)


def test_sample_seeded_key_is_deterministic(cuda):
    from ssd_b200.algorithm.verify import uniforms_from_seed, verify_sample

    lp, lq, spec, _, _ = _sample_inputs(4, 4, 5000, seed=5)
    r1 = verify_sample(lp, lq, spec, 1234)
    r2 = verify_sample(lp, lq, spec, 1234)
    assert r1.recovery_tokens.tolist() == r2.recovery_tokens.tolist()
    ua, ug = uniforms_from_seed(1234, 4, 4, 5000, "cuda")
    u = ug.cpu().numpy()
    assert (u > 0).all() and (u < 1).all() and abs(u.mean() - 0.5) < 0.01
    r3 = verify_sample(lp, lq, spec, (ua, ug))
    assert r3.recovery_tokens.tolist() == r1.recovery_tokens.tolist()


def _top_p_rows(v, seed, n=6):
    rng = np.random.default_rng(seed)
    rows = (3.0 * rng.standard_normal((max(n, 6), v))).astype(np.float32)
    rows[1] = np.round(rows[1] * 4) / 4                 # many ties
    rows[2, ::7] = -np.inf                              # already masked entries
    rows[2, 5] = np.nan
    rows[3] = np.float32(0.5)                           # all equal
    rows[4, 17] = 40.0                                  # one dominant logit
    return rows


@pytest.mark.parametrize("v,t,p,n", [(256000, 1.0, 0.95, 6), (256000, 0.7, 0.5, 6), (32000, 1.3, 0.9, 6),
                                     (4099, 1.0, 1e-4, 6), (32000, 1.0, 0.95, 80), (4099, 0.8, 0.7, 75)])
def test_top_p_mask_matches_oracle(cuda, v, t, p, n):
    """ssd_top_p_mask keeps exactly the oracle's nucleus (same values, everything else -inf); up to 74
    rows run four CTAs per row (a cluster), more rows one CTA per row."""
    import torch

    from oracle.verify import top_p_mask as o_mask
    from ssd_b200.algorithm.verify import top_p_mask_

    rows = _top_p_rows(v, seed=v + int(100 * p), n=n)
    got = top_p_mask_(torch.from_numpy(rows).cuda(), t, p).cpu().numpy()
    want = o_mask(rows, t, p)
    np.testing.assert_array_equal(got, want)
    kept = np.isfinite(want).sum(-1)
    assert (kept >= 1).all() and kept[3] == v  # ties: the all-equal row keeps every logit


@pytest.mark.parametrize("b,k,v", [(6, 6, 32000), (4, 4, 256000)])
def test_sample_with_top_p_matches_oracle(cuda, b, k, v):
    """Rejection sampling on the top-p nuclei (standard alignment, T = 1, p = 0.95) equals the oracle run
    on the oracle-masked logits with the same uniforms (near-ties excepted, as for plain sampling)."""
    from oracle.verify import top_p_mask as o_mask
    from ssd_b200.algorithm.verify import verify_sample

    lp, lq, spec, ua, ug = _sample_inputs(b, k, v, seed=7 * b + v)
    res = verify_sample(lp, lq, spec, (ua, ug), alignment="standard", top_p=0.95)
    acc, rec, mask, (am, gap) = o_sample(o_mask(lp, 1.0, 0.95), o_mask(lq, 1.0, 0.95), spec, ua, ug,
                                         alignment="standard", return_margins=True)
    ga = res.accept_until.cpu().numpy()
    gr = res.recovery_tokens.cpu().numpy()
    assert np.all((ga == acc) | (am < 1e-5)), (ga, acc, am)
    ok_rows = ga == acc
    assert np.all((gr == rec) | (gap < 1e-4) | ~ok_rows), (gr, rec, gap)
    # the recovery token lies inside the target's nucleus, or the draft's when every draft token was accepted
    lpm = o_mask(lp, 1.0, 0.95)
    for i in range(b):
        row = lpm[i, k] if ga[i] == k else lpm[i, ga[i]]
        assert np.isfinite(row[gr[i]])
