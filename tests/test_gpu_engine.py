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
    assert llm._engine.draft_device == torch.device("cuda", 1) and llm._engine.draft.dev == torch.device("cuda", 1)
    out, m = llm.generate([prompt], sampling)
    llm.shutdown()
    assert out[0] == ref[0] and m.total_tokens > 0


def test_adapter_built_from_a_model_path(cuda):
    """The reference's construction forms (gemma_adapter.py:28-36): by keyword and by position.
    With SSD_USE_TOY_MODEL set (tests/conftest.py), a path that names no preset gives the toy
    model of the role, and the second positional argument is the vocabulary size (ignored:
    the vocabulary comes from the weights), never a cache size."""
    from ssd_b200.models.gemma import PRESETS
    from ssd_b200.models.gemma_adapter import GemmaAdapter

    a = GemmaAdapter(model_path="toy-target", role="target")
    b = GemmaAdapter("some/checkpoint/dir", 256000)
    assert a.w.shape == b.w.shape == PRESETS["toy-target"]
    assert b.vocab_size == PRESETS["toy-target"].vocab and b.max_model_len == 4096
    prompt = torch.tensor(list(range(3, 20)))
    ra, rb = a.prefill(prompt), b.prefill(prompt)
    torch.testing.assert_close(ra.logits, rb.logits, rtol=0, atol=0)
    da = a.decode(int(ra.logits[0].argmax()))
    assert 0 <= da.next_token < a.vocab_size


def _tp_pair_config(mode, **kw):
    from ssd_b200 import DecodeMode, SSDConfig

    return SSDConfig(mode=DecodeMode(mode), target_model_path="tp-target", draft_model_path="tp-draft",
                     use_toy_model=False, **kw)


def test_engine_batches_several_prompts(cuda):
    """sd with several prompts runs them through the batched decoder, 4 rows at a time with
    refills (continuous batching); every stream equals the prompt's own AR stream."""
    from ssd_b200 import LLM, SamplingParams

    rng = np.random.default_rng(3)
    prompts = [[int(x) for x in rng.integers(0, 2048, n)] for n in (9, 40, 3, 77, 21, 55)]
    sampling = SamplingParams(max_new_tokens=14)
    ar = LLM(_tp_pair_config("ar"))
    refs = [ar.generate([p], sampling)[0][0] for p in prompts]
    ar.shutdown()
    llm = LLM(_tp_pair_config("sd", batch_buckets=(1, 2, 4)))
    got, m = llm.generate(prompts, sampling)
    llm.shutdown()
    assert got == refs
    # as in the reference's metrics, the first token of a sequence (the prefill's argmax) is not
    # counted in a step
    assert m.total_tokens == 6 * 13 and max(s.sequences for s in m.steps) == 4
    # sampling (temperature > 0) also takes the batched path: reproducible for the engine's seed
    llm = LLM(_tp_pair_config("sd"))
    hot = SamplingParams(max_new_tokens=10, temperature=1.0, top_p=0.9)
    a, _ = llm.generate(prompts[:3], hot)
    b, _ = llm.generate(prompts[:3], hot)
    llm.shutdown()
    assert a == b and all(len(x) == 10 for x in a)


def test_engine_tensor_parallel_modes(cuda):
    """The engine's target sharded over 2 GPUs in one process (one thread per GPU): sd and ssd
    reproduce the sharded AR stream; in ssd mode the draft runs on the next GPU when there is one."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from ssd_b200 import LLM, SamplingParams

    prompt = list(range(100, 160))
    sampling = SamplingParams(max_new_tokens=24)
    outs = {}
    for mode in ("ar", "sd", "ssd"):
        llm = LLM(_tp_pair_config(mode, tensor_parallel_size=2, fan_out_list=(3, 3, 3, 3, 3)))
        if mode == "ssd":
            want = torch.device("cuda", 2) if torch.cuda.device_count() > 2 else torch.device("cuda", 0)
            assert llm._engine.draft_device == want
        out, m = llm.generate([prompt], sampling)
        if mode == "sd":
            two, _ = llm.generate([prompt, prompt[:30]], sampling)  # batched, sharded
            assert two[0] == out[0]
        llm.shutdown()
        outs[mode] = out[0]
        assert len(out[0]) == 24 and m.total_tokens >= 23  # sd/ssd do not count the prefill token
    assert outs["ar"] == outs["sd"] == outs["ssd"]
