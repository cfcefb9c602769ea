"""Oracle (test infrastructure only): the reference's context-free toy model.

Restates ``ToyModelAdapter._logits_from_tokens`` of jax_ssd/models/toy_model.py:13-41
per call, as the reference computes it: for each token t a vector h that is zero
except h[t % H] = 1.0 and then h[(7 t) % H] = 0.5, times W, where
W = default_rng(seed).standard_normal((H, V)) in fp32, times 0.1.  Draft
speculation (toy_model.py:82-96) feeds the last token and takes the first-index
argmax k times.
"""

from __future__ import annotations

import numpy as np


def toy_weights(vocab_size: int = 64, hidden_dim: int = 32, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((hidden_dim, vocab_size)).astype(np.float32) * 0.1


def toy_logits(token_ids, w: np.ndarray) -> np.ndarray:
    """Logits [len, V] fp32 of the tokens (toy_model.py:33-41)."""
    hidden_dim = w.shape[0]
    ids = np.array(token_ids, dtype=np.int32).reshape(-1)
    h = np.zeros((len(ids), hidden_dim), dtype=np.float32)
    for i, t in enumerate(ids):
        h[i, t % hidden_dim] = 1.0
        h[i, (t * 7) % hidden_dim] = 0.5
    return h @ w


def toy_draft(prefix_tokens, k: int, w: np.ndarray):
    """(k greedy tokens, their logits [k, V]) after the prefix (toy_model.py:82-96)."""
    tokens = list(int(t) for t in prefix_tokens)
    rows = []
    for _ in range(k):
        lg = toy_logits(tokens[-1:], w)
        rows.append(lg[0])
        tokens.append(int(np.argmax(lg[0])))
    return tokens[len(tokens) - k:], np.stack(rows)
