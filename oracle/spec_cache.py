"""Oracle: speculation-cache lookup (test infrastructure only).

Restates ``jax_ssd/algorithm/spec_cache.py:43-66`` of the reference: a request
key ``[seq_id, accepted_index, recovery_token]`` hits the FIRST valid slot whose
key matches all three fields (``argmax`` over the match vector); a miss returns
index -1 and zero tokens/logits.  Pinned to ``tests/test_spec_cache.py:6-20``.
"""

from __future__ import annotations

import numpy as np


def lookup(keys, tokens, logits, valid, request_keys):
    """keys[N,3], tokens[N,K], logits[N,K,V], valid[N]; request_keys[B,3]."""
    m = np.all(request_keys[:, None, :] == keys[None, :, :], axis=-1) & valid[None, :]
    hit = m.any(-1)
    idx = np.where(hit, m.astype(np.int32).argmax(-1), -1).astype(np.int32)
    safe = np.maximum(idx, 0)
    tok = np.where(hit[:, None], tokens[safe], 0).astype(np.int32)
    lg = np.where(hit[:, None, None], logits[safe], 0).astype(np.float32)
    return hit, idx, tok, lg
