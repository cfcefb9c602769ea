"""GPU: the allocation-free greedy acceptance entry point (ssd_verify_greedy_noalloc).

Some callers of this library cannot call cudaMalloc: an XLA custom call is
handed only its operands and no allocator, and some embedders run under a
fixed device-memory budget.  For them
the library keeps the scratch of this one entry point in its own device data.
This test calls it through the C ABI and checks that its outputs equal those
of ssd_verify_greedy (which takes a caller workspace) on three calls in a row --
the later calls reuse the shared scratch the first one left behind.  The
outputs are integers, so the comparison is exact.  The file is named so that
pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(seed, b, k, v):
    rng = np.random.default_rng(seed)
    lp = (3.0 * rng.standard_normal((b, k + 1, v))).astype(np.float32)
    t = lp.argmax(-1)
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    for i in range(b):
        a = i % (k + 1)
        spec[i, 1:a + 1] = t[i, :a]
    return lp, spec


def test_noalloc_greedy_equals_workspace_entry_point(cuda):
    import torch

    from ssd_b200 import _lib
    from ssd_b200.algorithm.verify import verify_greedy

    so = _lib.lib()
    # the third call is the largest shape the fixed scratch takes: B * (K + 1) = 512 rows
    for call, (b, k, v) in enumerate([(8, 4, 256000), (6, 6, 32000), (8, 63, 32000)]):
        lp, spec = _inputs(call, b, k, v)
        ref, ref_tt = verify_greedy(lp, spec, target_tokens=True)
        d_lp = torch.tensor(lp, device="cuda")
        d_spec = torch.tensor(spec, device="cuda")
        acc = torch.full((b,), -7, dtype=torch.int32, device="cuda")
        rec = torch.full((b,), -7, dtype=torch.int32, device="cuda")
        mask = torch.full((b, k + 1), 9, dtype=torch.uint8, device="cuda")
        tt = torch.full((b, k + 1), -7, dtype=torch.int32, device="cuda")
        rc = so.ssd_verify_greedy_noalloc(_lib.stream_ptr(), d_lp.data_ptr(), d_spec.data_ptr(), acc.data_ptr(),
                                          rec.data_ptr(), mask.data_ptr(), tt.data_ptr(), b, k, v)
        assert rc == 0, _lib.lib().ssd_status_string(rc)
        torch.cuda.synchronize()
        assert torch.equal(acc, ref.accept_until)
        assert torch.equal(rec, ref.recovery_tokens)
        assert torch.equal(mask.bool(), ref.accepted_mask)
        assert torch.equal(tt, ref_tt)


def test_noalloc_greedy_rejects_sizes_over_its_limit(cuda):
    from ssd_b200 import _lib

    so = _lib.lib()
    # B * (K + 1) = 520 > 512: refused on the host before any launch
    assert so.ssd_verify_greedy_noalloc(_lib.stream_ptr(), 1, 1, 1, 1, None, None, 104, 4, 1000) == 4
