"""The reference's context-free toy model (jax_ssd/models/toy_model.py) on the device.

CPU: the oracle equals the golden vectors that the reference's own
``ToyModelAdapter`` produced (``tests/golden/make_golden.py``), and the H logit
rows the adapter keeps equal both, bit for bit.  GPU: prefill / decode /
verify / draft_speculate of ``ToyModelAdapter`` through ``ssd_embed`` and
``ssd_argmax_rows`` equal the oracle's, bit for bit.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle.toy_model import toy_draft, toy_logits, toy_weights

GOLDEN = Path(__file__).resolve().parent / "golden" / "toy_model.npz"


@pytest.mark.parametrize("vocab,hidden,seed", [(64, 32, 0), (100, 32, 3), (64, 16, 7)])
def test_toy_oracle_and_rows_match_reference_goldens(vocab, hidden, seed):
    from ssd_b200.models.toy_model import toy_logit_rows

    z = np.load(GOLDEN)
    name = f"v{vocab}_h{hidden}_s{seed}"
    ids = z[f"{name}__ids"]
    w = toy_weights(vocab, hidden, seed)
    np.testing.assert_array_equal(toy_logits(ids, w), z[f"{name}__logits"])
    np.testing.assert_array_equal(toy_logit_rows(vocab, hidden, seed)[ids % hidden], z[f"{name}__logits"])
    spec, lg = toy_draft(z[f"{name}__draft_prefix"], 5, w)
    assert spec == z[f"{name}__draft_spec"].tolist()
    np.testing.assert_array_equal(lg, z[f"{name}__draft_logits"])


@pytest.mark.parametrize("vocab,hidden,seed", [(64, 32, 0), (100, 32, 3), (64, 16, 7)])
def test_toy_rows_equal_reference_logits(vocab, hidden, seed):
    from ssd_b200.models.toy_model import toy_logit_rows

    w = toy_weights(vocab, hidden, seed)
    rows = toy_logit_rows(vocab, hidden, seed)
    ids = np.concatenate([np.arange(3 * hidden), np.random.default_rng(seed).integers(0, 10 * vocab, 50)])
    ref = toy_logits(ids, w)
    np.testing.assert_array_equal(rows[ids % hidden], ref)


@pytest.mark.gpu
@pytest.mark.parametrize("vocab,hidden,seed", [(64, 32, 0), (100, 32, 3)])
def test_toy_adapter_matches_reference(cuda, vocab, hidden, seed):
    from ssd_b200.models.toy_model import ToyModelAdapter

    w = toy_weights(vocab, hidden, seed)
    ad = ToyModelAdapter(vocab_size=vocab, hidden_dim=hidden, seed=seed)
    ids = np.random.default_rng(seed).integers(0, 3 * vocab, 9).astype(np.int32)
    pre = ad.prefill(ids, ad.allocate_kv(), None)
    np.testing.assert_array_equal(pre.logits.cpu().numpy(), toy_logits(ids, w))
    ver = ad.verify(ids[:5], None, None, None)
    assert tuple(ver.logits.shape) == (1, 5, vocab)
    np.testing.assert_array_equal(ver.logits[0].cpu().numpy(), toy_logits(ids[:5], w))
    dec = ad.decode(int(ids[0]), 0, None, None)
    assert dec.next_token == int(np.argmax(toy_logits(ids[:1], w)[0]))
    spec, lg = ad.draft_speculate([int(t) for t in ids], 4)
    ref_spec, ref_lg = toy_draft(ids, 4, w)
    assert spec == ref_spec
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_lg)
    assert ad.tokenize("hello") == [ord(c) % vocab for c in "hello"]
