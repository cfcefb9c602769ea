"""Engine, adapter and speculation-cache tests through the public API.

Mirrors the reference's ``tests/test_engine_modes.py:8-32`` (strengthened from
equal lengths to equal tokens) and ``tests/test_spec_cache.py:6-20`` (known
answers in ``tests/golden/spec_cache.json``).  Every call runs the CUDA library.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def test_spec_cache_known_answers(cuda):
    from ssd_b200.algorithm.spec_cache import SpecCache

    for name, case in json.loads((GOLDEN / "spec_cache.json").read_text()).items():
        cache = SpecCache.create(num_branches=case["num_branches"], k=case["k"], vocab=case["vocab"], device=cuda)
        for ins in case["inserts"]:
            cache = cache.insert(ins["slot"], ins["key"], ins["tokens"],
                                 torch.zeros((case["k"], case["vocab"])))
        for lk in case["lookups"]:
            hit, idx, tok, lg = cache.lookup(torch.tensor([lk["key"]], dtype=torch.int32))
            assert bool(hit[0]) == lk["hit"], name
            assert int(idx[0]) == lk["idx"], name
            if lk["hit"]:
                assert tok[0].tolist() == lk["tokens"], name


def test_spec_cache_first_match_and_logits_vs_oracle(cuda):
    """Random keys with duplicates: hit / first matching slot / gathered rows equal the oracle."""
    from oracle import spec_cache as osc
    from ssd_b200.algorithm.spec_cache import SpecCache

    rng = np.random.default_rng(7)
    n, k, v = 64, 6, 48
    keys = rng.integers(0, 4, size=(n, 3)).astype(np.int32)
    tokens = rng.integers(0, v, size=(n, k)).astype(np.int32)
    logits = rng.standard_normal((n, k, v)).astype(np.float32)
    valid = rng.random(n) < 0.7
    cache = SpecCache.create(n, k, v, device=cuda)
    for s in range(n):
        if valid[s]:
            cache.insert(s, keys[s], tokens[s], logits[s])
    req = rng.integers(0, 5, size=(40, 3)).astype(np.int32)
    hit, idx, tok, lg = cache.lookup(req)
    rh, ri, rt, rl = osc.lookup(keys, tokens, logits, valid, req)
    np.testing.assert_array_equal(hit.cpu().numpy(), rh)
    np.testing.assert_array_equal(idx.cpu().numpy()[rh], np.asarray(ri)[rh])
    np.testing.assert_array_equal(tok.cpu().numpy()[rh], np.asarray(rt)[rh])
    np.testing.assert_array_equal(lg.cpu().numpy()[rh], np.asarray(rl)[rh])
    assert (idx.cpu().numpy()[~rh] == -1).all()


def test_ar_generates_tokens(cuda):
    from ssd_b200 import LLM, DecodeMode, SamplingParams

    llm = LLM.from_mode(DecodeMode.AR)
    outputs, metrics = llm.generate([[1, 2, 3, 4, 5]], SamplingParams(max_new_tokens=8))
    llm.shutdown()
    assert len(outputs[0]) == 8
    assert metrics.total_tokens > 0


def test_sd_ssd_greedy_equal_tokens_to_ar(cuda):
    """The three modes emit the same greedy stream (the reference asserts equal lengths)."""
    from ssd_b200 import LLM, DecodeMode, SamplingParams

    prompt = [10, 20, 30]
    sampling = SamplingParams(max_new_tokens=12)
    outs = {}
    for mode in (DecodeMode.AR, DecodeMode.SD, DecodeMode.SSD):
        llm = LLM.from_mode(mode)
        out, m = llm.generate([prompt], sampling)
        llm.shutdown()
        outs[mode] = out[0]
        assert m.total_tokens > 0
    assert len(outs[DecodeMode.AR]) == 12
    assert outs[DecodeMode.AR] == outs[DecodeMode.SD] == outs[DecodeMode.SSD]


def test_ssd_self_draft_hits_and_accepts(cuda):
    """Draft == target: every draft is accepted, the stream still equals AR, the cache is exercised."""
    from ssd_b200 import LLM, DecodeMode, SamplingParams, SSDConfig

    prompt = list(range(3, 40))
    sampling = SamplingParams(max_new_tokens=20)
    ar = LLM.from_mode(DecodeMode.AR)
    ref, _ = ar.generate([prompt], sampling)
    ar.shutdown()
    cfg = SSDConfig(mode=DecodeMode.SSD, target_model_path="toy-target", draft_model_path="toy-target",
                    use_toy_model=True)
    llm = LLM(cfg)
    out, m = llm.generate([prompt], sampling)
    out2, m2 = llm.generate([prompt], sampling)
    llm.shutdown()
    assert out[0] == ref[0] and out2[0] == ref[0]
    assert m.accepted_per_step > 1.5
    # every step after the first is served from the pre-drafted bonus branch
    assert m.cache_hit_rate > 0.5 and m2.cache_hit_rate > 0.5


def test_generate_strings_and_stream(cuda):
    from ssd_b200 import LLM, DecodeMode, SamplingParams

    llm = LLM.from_mode("sd")
    out, _ = llm.generate(["hello"], SamplingParams(max_new_tokens=6))
    got = []
    toks = [t for t, _ in llm.generate_stream("hello", SamplingParams(max_new_tokens=6),
                                               on_token=lambda t, s: got.append(t))]
    llm.shutdown()
    assert out[0] == toks == got and len(toks) == 6


def test_adapter_verify_commit_matches_prefill(cuda):
    """verify + commit leaves the cache as a prefill of the committed stream would."""
    from ssd_b200.models.gemma_adapter import GemmaAdapter
    from ssd_b200.models.model_loader import load_weights

    w = load_weights("toy-target", use_toy=True)
    a = GemmaAdapter(w, max_model_len=256)
    b = GemmaAdapter(w, max_model_len=256)
    prompt = list(range(5, 30))
    r = int(a.prefill(torch.tensor(prompt)).logits[0].argmax())
    spec = [7, 8, 9, 10]
    lg = a.verify(torch.tensor([r] + spec)).logits[0]
    # commit r + 2 drafts, new recovery 99
    a.commit_tokens(spec[:2] + [99])
    assert a.cached == prompt + [r] + spec[:2]
    pa = a.decode(99).logits
    pb = b.prefill(torch.tensor(prompt + [r] + spec[:2] + [99])).logits
    torch.testing.assert_close(pa, pb, rtol=0, atol=0)
    # the verify logits of position 0 equal a decode of r after the prompt
    c = GemmaAdapter(w, max_model_len=256)
    c.prefill(torch.tensor(prompt))
    torch.testing.assert_close(c.decode(r).logits[0], lg[0], rtol=0, atol=0)


def test_ssd_draft_on_its_own_gpu(cuda):
    """ssd mode with the draft model and its worker on a second GPU: same stream as AR."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from ssd_b200 import LLM, DecodeMode, SamplingParams, SSDConfig

    prompt = list(range(7, 30))
    sampling = SamplingParams(max_new_tokens=16)
    ar = LLM.from_mode(DecodeMode.AR)
    ref, _ = ar.generate([prompt], sampling)
    ar.shutdown()
    llm = LLM(SSDConfig(mode=DecodeMode.SSD, use_toy_model=True, draft_device="cuda:1"))
    assert llm._engine.draft_w.device == torch.device("cuda", 1)
    out, m = llm.generate([prompt], sampling)
    llm.shutdown()
    assert out[0] == ref[0] and m.total_tokens > 0
