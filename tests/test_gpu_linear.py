"""GPU numerics: skinny projections (K3) with fused epilogues vs a plain fp32 reference."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.gemma import bf16_round, gelu_tanh

pytestmark = pytest.mark.gpu


def _bf16_close(got, exp, ulps=1.0, atol=1e-6):
    """|got - exp| within `ulps` bf16 ulps of |exp| (fp32 accumulation order differs).

    A bf16 ulp is 2^(e-7) for |x| in [2^e, 2^(e+1)), i.e. at most |x| * 2^-7.
    """
    tol = np.abs(exp) * (2.0 ** -7) * ulps + atol
    bad = np.abs(got - exp) > tol
    assert not bad.any(), (np.abs(got - exp)[bad][:5], exp[bad][:5])


@pytest.mark.parametrize("m,n,k", [(5, 12288, 3072), (1, 3072, 4096), (5, 3072, 24576), (16, 1000, 512),
                                   (7, 2048, 2048)])
def test_store_bf16(cuda, m, n, k):
    import torch

    from ssd_b200.kernels.ops import linear

    g = torch.Generator(device="cuda").manual_seed(m * n + k)
    x = torch.randn((m, k), device="cuda", generator=g).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / k ** 0.5).bfloat16()
    y = linear(x, w, "store")
    ref = (x.float() @ w.float().T).cpu().numpy()  # plain PyTorch fp32 reference
    _bf16_close(y.float().cpu().numpy(), bf16_round(ref), ulps=1.0, atol=1e-3)


def test_store_f32_logits(cuda):
    import torch

    from ssd_b200.kernels.ops import linear

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn((5, 3072), device="cuda", generator=g).bfloat16()
    w = (0.005 * torch.randn((256000, 3072), device="cuda", generator=g)).bfloat16()
    y = linear(x, w, "store_f32")
    ref = x.float() @ w.float().T
    assert y.dtype == torch.float32
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-4)


def test_residual_and_geglu(cuda):
    import torch

    from ssd_b200.kernels.ops import linear

    g = torch.Generator(device="cuda").manual_seed(1)
    m, d, f = 5, 3072, 24576
    x = torch.randn((m, d), device="cuda", generator=g).bfloat16()
    wgu = (torch.randn((2 * f, d), device="cuda", generator=g) / d ** 0.5).bfloat16()
    a = linear(x, wgu, "geglu")
    assert a.shape == (m, f)
    acc = (x.float() @ wgu.float().T).cpu().numpy()
    gate, up = bf16_round(acc[:, 0::2]), bf16_round(acc[:, 1::2])
    exp = bf16_round(bf16_round(gelu_tanh(gate)) * up)
    # the gate/up accumulators may round differently by one bf16 ulp; compare loosely then on average
    got = a.float().cpu().numpy()
    assert np.abs(got - exp).max() < 0.05
    assert np.mean(got == exp) > 0.97
    wd = (torch.randn((d, f), device="cuda", generator=g) / f ** 0.5).bfloat16()
    res = torch.randn((m, d), device="cuda", generator=g).bfloat16()
    res0 = res.clone()
    linear(a, wd, "residual", out=res)
    acc2 = bf16_round((a.float() @ wd.float().T).cpu().numpy())
    exp2 = bf16_round(res0.float().cpu().numpy() + acc2)
    _bf16_close(res.float().cpu().numpy(), exp2, ulps=2.0, atol=2e-2)


@pytest.mark.parametrize("n,k", [(12288, 3072), (3072, 24576), (256000, 3072)])
def test_rows_are_batch_invariant(cuda, n, k):
    """Row i of an M-row projection equals the same row projected alone, bit for bit."""
    import torch

    from ssd_b200.kernels.ops import linear

    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn((5, k), device="cuda", generator=g).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / k ** 0.5).bfloat16()
    full = linear(x, w, "store_f32")
    for i in (0, 3, 4):
        one = linear(x[i:i + 1].contiguous(), w, "store_f32")
        assert torch.equal(one[0], full[i])


def test_fp32_weights_toy(cuda):
    import torch

    from ssd_b200.kernels.ops import linear

    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn((5, 256), device="cuda", generator=g)
    w = torch.randn((1024, 256), device="cuda", generator=g) * 0.06
    y = linear(x, w, "store")
    torch.testing.assert_close(y, x @ w.T, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("m,n,k", [(17, 1000, 520), (64, 3072, 3072), (200, 513, 1024), (256, 4096, 256),
                                   (5, 256000, 3072), (2, 130, 64)])
def test_tcgen05_shapes_and_tails(cuda, m, n, k):
    """M up to 256 (UMMA N = 16..256), N and K not multiples of the 128 x 64 tile."""
    import torch

    from ssd_b200.kernels.ops import linear
    from ssd_b200.workspace import workspace

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn((m, k), device="cuda", generator=g).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / k ** 0.5).bfloat16()
    y = linear(x, w, "store_f32", ws_key="tc_test")
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-4)
    torch.cuda.synchronize()
    ws = workspace(x.device, "tc_test", 0)
    head = ws[: 16384 * 4 + 4].view(torch.int32)
    assert int(head[:16384].abs().sum()) == 0      # ticket counters reset
    assert int(head[16384]) == 0                   # no device-side wait gave up


@pytest.mark.parametrize("dtype_name,m,n,k,epi", [("bf16", 5, 12288, 3072, "store"), ("bf16", 5, 2 * 24576, 3072, "geglu"),
                                                  ("bf16", 1, 2560, 2048, "store"), ("f32", 5, 1024, 256, "store"),
                                                  ("f32", 3, 2048, 256, "geglu"), ("bf16", 224, 12288, 3072, "store"),
                                                  ("bf16", 32, 2 * 16384, 2048, "geglu")])
def test_rownorm_projection(cuda, dtype_name, m, n, k, epi):
    """ssd_linear_rownorm = round(rsqrt(mean(x^2)+eps) * (x w^T)), the folded-norm projection."""
    import torch

    from ssd_b200.kernels.ops import linear

    dt = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(m * n)
    x = (3.0 * torch.randn((m, k), device="cuda", generator=g)).to(dt)
    w = (torch.randn((n, k), device="cuda", generator=g) / k ** 0.5).to(dt)
    y = linear(x, w, epi, rownorm_eps=1e-6)
    xf = x.float()
    inv = 1.0 / torch.sqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)
    acc = (xf @ w.float().T) * inv
    if epi == "geglu":
        gate, up = acc[:, 0::2], acc[:, 1::2]
        if dt == torch.bfloat16:
            gate, up = gate.bfloat16().float(), up.bfloat16().float()
        ref = torch.nn.functional.gelu(gate, approximate="tanh")
        if dt == torch.bfloat16:
            ref = ref.bfloat16().float()
        ref = ref * up
    else:
        ref = acc
    tol = 2e-2 if dt == torch.bfloat16 else 1e-5
    torch.testing.assert_close(y.float(), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("n,k", [(3072, 4096), (2048, 2048), (2560, 2048), (2048, 16384), (768, 2048), (3072, 128),
                                 (12288, 3072)])
def test_tile_split_rows_match_across_m(cuda, n, k):
    """Shapes with at most as many 128-row output tiles as SMs cut every tile's K range into G
    parts: for M <= 16 the G CTAs of a tile form one thread-block cluster and fold their partials in
    distributed shared memory, for larger M the same parts go through the global ticket fold.  Every
    row is bit-identical for M = 1, 5, 16, 40 and 224 (plain, row-norm and residual epilogues; above
    16 rows the row norms come from their own kernel, below from the projection's epilogue)."""
    import torch

    from ssd_b200.kernels.ops import linear
    from ssd_b200.workspace import workspace

    g = torch.Generator(device="cuda").manual_seed(n + k)
    x = (2.0 * torch.randn((224, k), device="cuda", generator=g)).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / k ** 0.5).bfloat16()
    res = torch.randn((224, n), device="cuda", generator=g).bfloat16()
    full = linear(x, w, "store_f32", ws_key="split_test")
    torch.testing.assert_close(full, x.float() @ w.float().T, rtol=1e-4, atol=1e-4)
    full_norm = linear(x, w, "store", rownorm_eps=1e-6, ws_key="split_test")
    full_res = res.clone()
    linear(x, w, "residual", out=full_res, ws_key="split_test")
    for m in (1, 5, 16, 40):
        assert torch.equal(linear(x[:m].contiguous(), w, "store_f32", ws_key="split_test"), full[:m])
        assert torch.equal(linear(x[:m].contiguous(), w, "store", rownorm_eps=1e-6, ws_key="split_test"),
                           full_norm[:m])
        r = res[:m].clone()
        linear(x[:m].contiguous(), w, "residual", out=r, ws_key="split_test")
        assert torch.equal(r, full_res[:m])
    torch.cuda.synchronize()
    head = workspace(x.device, "split_test", 0)[: 16384 * 4 + 4].view(torch.int32)
    assert int(head[:16384].abs().sum()) == 0      # ticket counters reset
    assert int(head[16384]) == 0                   # no device-side wait gave up
