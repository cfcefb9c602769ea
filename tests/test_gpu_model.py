"""GPU parity of the whole verify forward and of greedy speculative decoding.

Criteria (from the path's spec): logits within 1e-4 of the oracle in fp32 on the
toy pair and within 2e-2 in bf16 at Gemma-7B layer shapes; greedy token streams
identical on >= 99% of seeded prompts; SD stream == AR stream.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.gemma import GemmaShape as OShape
from oracle.gemma import OracleGemma, greedy_ar, new_pages

pytestmark = pytest.mark.gpu


def _oshape(s):
    return OShape(s.num_layers, s.d_model, s.num_heads, s.num_kv_heads, s.head_dim, s.ffn, s.vocab)


def _run_forward(w, prompt, verify_tokens, bs=16):
    """Prefill `prompt` in chunks, then one verify forward over `verify_tokens`; returns its logits."""
    import torch

    from ssd_b200.kernels.ops import max_tokens_per_forward
    from ssd_b200.models.gemma import GemmaRunner
    from ssd_b200.kernels.kv_cache import KVCacheState

    s = w.shape
    n = len(prompt) + len(verify_tokens)
    nb = (n + bs - 1) // bs + 1
    cache = KVCacheState.allocate(s.num_layers, nb, bs, s.num_kv_heads, s.head_dim, dtype=w.dtype)
    table = torch.arange(nb, dtype=torch.int32, device="cuda")[None]
    run = GemmaRunner(w, 1, 64, nb * bs)
    chunk = min(64, max_tokens_per_forward(w.dtype))
    p = torch.tensor([prompt], dtype=torch.int32, device="cuda")
    for c0 in range(0, len(prompt), chunk):
        c1 = min(len(prompt), c0 + chunk)
        run.forward(p[:, c0:c1].contiguous(), torch.tensor([c0], dtype=torch.int32, device="cuda"), cache.pages,
                    table, None, last_only=True)
    vt = torch.tensor([verify_tokens], dtype=torch.int32, device="cuda")
    lg = torch.empty((1, len(verify_tokens), s.vocab), dtype=torch.float32, device="cuda")
    run.forward(vt, torch.tensor([len(prompt)], dtype=torch.int32, device="cuda"), cache.pages, table, lg)
    torch.cuda.synchronize()
    return lg[0].cpu().numpy()


def _oracle_forward(w, prompt, verify_tokens, precision, layers=None, bs=16):
    shape = _oshape(w.shape)
    om = OracleGemma(shape, w.to_canonical(layers), precision)
    n = len(prompt) + len(verify_tokens)
    nb = (n + bs - 1) // bs + 1
    pages = new_pages(shape, nb, bs)
    table = np.arange(nb, dtype=np.int32)[None]
    om.forward(np.array([prompt]), pages, table, [0])
    return om.forward(np.array([verify_tokens]), pages, table, [len(prompt)])[0]


def test_toy_fp32_logits_within_1e4(cuda):
    import torch

    from ssd_b200.models.gemma import PRESETS, GemmaWeights

    w = GemmaWeights.random(PRESETS["toy-target"], seed=3, dtype=torch.float32)
    rng = np.random.default_rng(0)
    prompt = [int(x) for x in rng.integers(0, 1024, 64)]
    vt = [int(x) for x in rng.integers(0, 1024, 5)]
    got = _run_forward(w, prompt, vt)
    ref = _oracle_forward(w, prompt, vt, "fp32")
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=0)


def test_gemma7b_layer_shapes_bf16_logits_within_2e2(cuda):
    """Two decoder layers at the Gemma-7B widths (d 3072, 16x256 heads, FFN 24576), bf16."""
    import torch

    from ssd_b200.models.gemma import GemmaShape, GemmaWeights

    shape = GemmaShape(2, 3072, 16, 16, 256, 24576, 32768)
    w = GemmaWeights.random(shape, seed=7, dtype=torch.bfloat16)
    rng = np.random.default_rng(1)
    prompt = [int(x) for x in rng.integers(0, shape.vocab, 40)]
    vt = [int(x) for x in rng.integers(0, shape.vocab, 5)]
    got = _run_forward(w, prompt, vt)
    ref = _oracle_forward(w, prompt, vt, "bf16")
    err = np.abs(got - ref)
    assert err.max() < 2e-2, err.max()
    assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.8


def test_gemma2b_mqa_layer_shapes_bf16(cuda):
    import torch

    from ssd_b200.models.gemma import GemmaShape, GemmaWeights

    shape = GemmaShape(2, 2048, 8, 1, 256, 16384, 16384)
    w = GemmaWeights.random(shape, seed=8, dtype=torch.bfloat16)
    rng = np.random.default_rng(2)
    prompt = [int(x) for x in rng.integers(0, shape.vocab, 33)]
    vt = [int(x) for x in rng.integers(0, shape.vocab, 2)]
    got = _run_forward(w, prompt, vt)
    ref = _oracle_forward(w, prompt, vt, "bf16")
    assert np.abs(got - ref).max() < 2e-2


def _full_depth_verify_check(preset, seed, prompt_len, k):
    """One verify forward of the whole model (every layer, the full vocabulary) after a
    ``prompt_len``-token prompt, and the oracle's forward of the same weights in bf16 (rounding
    where the CUDA path stores bf16) and in fp32 (no intermediate rounding).  The oracle fetches
    one layer at a time from the device (``GemmaWeights.canonical_layer``), so host memory holds
    the embedding plus one layer."""
    import torch

    from ssd_b200.models.gemma import PRESETS, GemmaWeights

    shape = PRESETS[preset]
    w = GemmaWeights.random(shape, seed=seed, dtype=torch.bfloat16, max_pos=1024)
    rng = np.random.default_rng(seed)
    prompt = [int(x) for x in rng.integers(0, shape.vocab, prompt_len)]
    vt = [int(x) for x in rng.integers(0, shape.vocab, k + 1)]
    got = _run_forward(w, prompt, vt)
    full = w.to_canonical(layers=0)
    full["layers"] = w.canonical_layer
    refs = {}
    for precision in ("bf16", "fp32"):
        om = OracleGemma(_oshape(shape), full, precision, max_pos=1024)
        n = len(prompt) + len(vt)
        nb = (n + 15) // 16 + 1
        pages = new_pages(om.s, nb, 16)
        table = np.arange(nb, dtype=np.int32)[None]
        om.forward(np.array([prompt]), pages, table, [0], with_head=False)
        refs[precision] = om.forward(np.array([vt]), pages, table, [len(prompt)])[0]
    return got, refs["bf16"], refs["fp32"]


@pytest.mark.parametrize("preset,seed", [("gemma-7b", 1000), ("gemma-2b", 2000)])
def test_full_depth_verify_logits(cuda, preset, seed):
    """The benchmarked models at full depth: Gemma-7B (28 layers) and Gemma-2B (18 layers), vocab
    256000, verify over k+1 = 5 tokens after a 128-token prompt.

    The per-op bf16 tolerance (2e-2, met by the 2-layer tests above) does not bound the maximum over
    1.28 M logits after 28 layers: every bf16 rounding point of the forward can round an fp32 value
    that the GPU and the oracle summed in different orders to neighbouring bf16 values, and these
    one-ulp differences propagate through the residual stream.  So the full-depth criteria are
    stated against the fp32 forward of the same weights: the GPU must be as close to it as the bf16
    oracle is (within 1.5x, max and mean), the GPU-vs-bf16-oracle difference must stay small
    (max <= 5e-2, mean <= 1e-2, for logits of standard deviation ~0.25), and the greedy choice must
    agree on at least 4 of the 5 positions (a top-2 gap inside the rounding noise may flip one)."""
    got, ref, ref32 = _full_depth_verify_check(preset, seed, 128, 4)
    e16 = np.abs(got - ref)
    g32 = np.abs(got - ref32)
    o32 = np.abs(ref - ref32)
    print(f"{preset}: |GPU - bf16 oracle| max {e16.max():.3e} mean {e16.mean():.3e}; "
          f"|GPU - fp32| max {g32.max():.3e} mean {g32.mean():.3e}; "
          f"|bf16 oracle - fp32| max {o32.max():.3e} mean {o32.mean():.3e}; logit std {ref32.std():.3e}")
    assert g32.max() <= 1.5 * o32.max() and g32.mean() <= 1.5 * o32.mean()
    assert e16.max() <= 5e-2 and e16.mean() <= 1e-2
    assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.8 and (got.argmax(-1) == ref32.argmax(-1)).mean() >= 0.8


def test_toy_gpu_ar_stream_matches_oracle(cuda):
    """Greedy streams identical to the oracle's on >= 99% of seeded prompts (toy pair, fp32)."""
    import torch

    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.runtime.speculative import GreedyDecoder

    w = GemmaWeights.random(PRESETS["toy-target"], seed=0, dtype=torch.float32)
    om = OracleGemma(_oshape(w.shape), w.to_canonical(), "fp32")
    dec = GreedyDecoder(w, max_seq_len=256)
    same = 0
    n_prompts = 20
    for s in range(n_prompts):
        prompt = [int(x) for x in np.random.default_rng(100 + s).integers(0, 1024, 64)]
        got = GreedyDecoder(w, max_seq_len=256).generate(prompt, 32) if s else dec.generate(prompt, 32)
        same += got == greedy_ar(om, prompt, 32)
    assert same / n_prompts >= 0.99


@pytest.mark.parametrize("draft_kind", ["independent", "self"])
def test_toy_sd_stream_equals_ar_stream(cuda, draft_kind):
    import torch

    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.runtime.speculative import GreedyDecoder, SpeculativeDecoder

    t = GemmaWeights.random(PRESETS["toy-target"], seed=0, dtype=torch.float32)
    d = t if draft_kind == "self" else GemmaWeights.random(PRESETS["toy-draft"], seed=1, dtype=torch.float32)
    for s in range(4):
        prompt = [int(x) for x in np.random.default_rng(s).integers(0, 1024, 64)]
        ar = GreedyDecoder(t, max_seq_len=512).generate(prompt, 128)
        sd, info = SpeculativeDecoder(t, d, k=4, max_seq_len=512).generate(prompt, 128)
        assert sd == ar
        if draft_kind == "self":
            assert info["steps"] <= 128 // 5 + 1  # every draft token accepted


def test_gemma_7b_2b_sd_equals_ar_bf16(cuda):
    """Full-size random-init Gemma-7B target / Gemma-2B draft: SD greedy stream == AR stream."""
    import torch

    from ssd_b200.models.gemma import PRESETS, GemmaWeights
    from ssd_b200.runtime.speculative import GreedyDecoder, SpeculativeDecoder

    t = GemmaWeights.random(PRESETS["gemma-7b"], seed=11)
    d = GemmaWeights.random(PRESETS["gemma-2b"], seed=12)
    prompt = [int(x) for x in np.random.default_rng(5).integers(0, 256000, 128)]
    ar = GreedyDecoder(t, max_seq_len=512).generate(prompt, 24)
    sd, _ = SpeculativeDecoder(t, d, k=4, max_seq_len=512).generate(prompt, 24)
    assert sd == ar
    sd2, info = SpeculativeDecoder(t, t, k=4, max_seq_len=512).generate(prompt, 24)
    assert sd2 == ar and info["steps"] <= 24 // 5 + 1
    del t, d
    torch.cuda.empty_cache()


@pytest.mark.parametrize("shape_args", [(2, 3072, 16, 16, 256, 24576, 32768), (2, 2048, 8, 1, 256, 16384, 16384)])
def test_rope_in_qkv_epilogue_equals_separate_rope(cuda, shape_args):
    """bf16 weights store each q/k head's rows as rotation pairs and the QKV projection applies RoPE and
    writes the K/V rows in its epilogue; the same weights in canonical order run the plain projection and
    the separate RoPE + K/V write kernel (prefill chunks and a 5-token verify forward).

    Pairing moves rows between the two 128-row tiles of a 256-wide head.  Where every tile is cut at the
    same k-blocks (the tile-split plan: Gemma-2B's 20-tile QKV) a row's sums do not depend on its tile, so
    logits and the whole K/V cache are bit-identical.  Gemma-7B's 96-tile QKV runs stream-K, whose split
    points differ between tiles, so there the two orders round differently: the logits agree within the
    bf16 criterion of the oracle tests and the K/V rows within a few bf16 ulps."""
    import torch

    from ssd_b200.kernels.kv_cache import KVCacheState
    from ssd_b200.models.gemma import GemmaRunner, GemmaShape, GemmaWeights

    shape = GemmaShape(*shape_args)
    plain = GemmaWeights.random(shape, seed=12, dtype=torch.bfloat16, max_pos=512)
    assert not plain.qk_pairs
    fused = GemmaWeights.from_canonical(shape, plain.to_canonical(), dtype=torch.bfloat16, max_pos=512,
                                        qk_pairs=True)
    assert fused.qk_pairs
    assert all(np.array_equal(a["wq"], b["wq"]) and np.array_equal(a["wk"], b["wk"])
               for a, b in zip(fused.to_canonical()["layers"], plain.to_canonical()["layers"]))
    rng = np.random.default_rng(5)
    prompt = torch.tensor([[int(x) for x in rng.integers(0, shape.vocab, 70)]], dtype=torch.int32, device=cuda)
    vt = torch.tensor([[int(x) for x in rng.integers(0, shape.vocab, 5)]], dtype=torch.int32, device=cuda)
    outs = []
    for w in (fused, plain):
        cache = KVCacheState.allocate(shape.num_layers, 8, 16, shape.num_kv_heads, shape.head_dim,
                                      dtype=torch.bfloat16)
        cache.pages.zero_()
        table = torch.arange(8, dtype=torch.int32, device=cuda)[None]
        run = GemmaRunner(w, 1, 64, 128)
        for c0 in (0, 64):
            c1 = min(70, c0 + 64)
            run.forward(prompt[:, c0:c1].contiguous(), torch.tensor([c0], dtype=torch.int32, device=cuda),
                        cache.pages, table, None, last_only=True)
        lg = torch.empty((1, 5, shape.vocab), dtype=torch.float32, device=cuda)
        run.forward(vt, torch.tensor([70], dtype=torch.int32, device=cuda), cache.pages, table, lg)
        torch.cuda.synchronize()
        outs.append((lg.clone(), cache.pages.clone()))
    tile_split = (shape.num_heads + 2 * shape.num_kv_heads) * shape.head_dim // 128 * 2 <= 148
    if tile_split:
        assert torch.equal(outs[0][0], outs[1][0])
        assert torch.equal(outs[0][1], outs[1][1])
    else:
        assert (outs[0][0] - outs[1][0]).abs().max().item() < 2e-2
        # layer 0 sees identical inputs on both paths: its K/V rows differ only where the two summation
        # orders round a q/k value to different bf16 neighbours (rare, one ulp of the inputs); later layers
        # inherit those differences through attention and the MLP
        k0 = (outs[0][1][:, 0].float() - outs[1][1][:, 0].float()).abs()
        ref0 = outs[1][1][:, 0].float().abs()
        assert (k0 > 0).float().mean().item() < 1e-3
        assert bool((k0 <= ref0 * 2.0 ** -6 + 2.0 ** -6).all())
