"""Oracle: greedy speculative decoding loop on the oracle Gemma (test infrastructure only).

Follows the sd loop of ``jax_ssd/runtime/engine.py:213-254`` — each step
verifies ``[recovery] + draft[k]`` with the target, applies ``verify_greedy``
and appends ``accepted + [recovery]`` — with the KV bookkeeping done the way a
correct cache-based verify needs it (the reference re-runs one forward per
committed token instead, ``gemma_adapter.py:145-152``): the verify pass writes
the k+1 new K/V rows, and the target's sequence length is then cut back to
``old + 1 + accepted``.  Output is truncated to ``max_new`` tokens.
"""

from __future__ import annotations

import numpy as np

from .gemma import OracleGemma, new_pages
from .verify import verify_greedy


def greedy_sd(target: OracleGemma, draft: OracleGemma, prompt, max_new: int, k: int = 4,
              num_blocks: int = 64, block_size: int = 16):
    tp = new_pages(target.s, num_blocks, block_size)
    dp = new_pages(draft.s, num_blocks, block_size)
    table = np.arange(num_blocks, dtype=np.int32)[None, :]
    seq = list(int(t) for t in prompt)
    lg = target.forward(np.array([seq]), tp, table, [0])
    out = [int(np.argmax(lg[0, -1]))]
    seq.append(out[-1])
    n_t = len(prompt)          # tokens in the target cache
    draft.forward(np.array([seq[:-1]]), dp, table, [0])
    n_d = len(prompt)          # tokens in the draft cache
    steps = 0
    while len(out) < max_new:
        feed = seq[n_d:]
        spec = []
        for _ in range(k):
            lgd = draft.forward(np.array([feed]), dp, table, [n_d])
            n_d += len(feed)
            spec.append(int(np.argmax(lgd[0, -1])))
            feed = [spec[-1]]
        vt = target.forward(np.array([[seq[-1]] + spec]), tp, table, [n_t])
        acc, rec, _ = verify_greedy(vt, np.array([[seq[-1]] + spec], np.int32))
        a, r = int(acc[0]), int(rec[0])
        new = spec[:a] + [r]
        n_t = n_t + 1 + a
        n_d = len(seq) + min(a, k - 1)
        out.extend(new)
        seq.extend(new)
        steps += 1
    return out[:max_new], steps
