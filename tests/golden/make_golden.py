"""Generate golden vectors by running the reference's own importable code.

Two pieces of the reference run without JAX and are executed here directly:

* ``reference/cuda_ssd/verify_torch.py`` (``verify_greedy_torch``) — the greedy
  accept/recovery rule of ``jax_ssd/algorithm/verify.py:18-59`` restated in
  torch by the reference itself; its parity test is
  ``tests/test_verify_parity.py:13-25`` (seed 42, standard-normal logits).
* ``jax_ssd/runtime/page_manager.py`` + ``jax_ssd/runtime/sequence.py`` — the
  host page allocator with its LIFO free list and ref counts.  They are loaded
  by file path with stub parent packages so that ``jax_ssd/__init__.py`` (which
  imports jax) is skipped.

The known answers of ``tests/test_spec_cache.py:6-20`` (JAX, not importable
here) are transcribed as a small case list.

``jax_ssd/models/toy_model.py`` (``ToyModelAdapter``) computes its logits in
numpy and only wraps them with ``jax.numpy`` (``array``, ``argmax``, ``stack``).
It is loaded by file path, with ``jax`` / ``jax.numpy`` replaced by a numpy
stand-in for those three calls (plus the names that its imports only mention:
``jnp.bfloat16`` as a default argument, ``jax.Array`` in annotations), so the
reference's own code produces the toy golden vectors.

Usage (from the repository root, with the reference checkout available)::

    python tests/golden/make_golden.py /path/to/reference

Writes ``tests/golden/verify_greedy.npz``, ``tests/golden/page_manager.json``,
``tests/golden/spec_cache.json`` and ``tests/golden/toy_model.npz``.
GPU test runs never execute this script; they read the committed fixtures.
"""

from __future__ import annotations

import importlib.util
import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def greedy_cases():
    """Seeded greedy-verify inputs: the reference test's shapes plus edge cases."""
    cases = []
    # tests/test_verify_parity.py:13-25 -- one rng(42) per shape
    for b, k, v in [(1, 4, 32), (4, 4, 64), (2, 8, 128)]:
        rng = np.random.default_rng(42)
        lp = rng.standard_normal((b, k + 1, v)).astype(np.float32)
        spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
        cases.append((f"ref_b{b}_k{k}_v{v}", lp, spec))
    # all accepted / partially accepted rows built from the argmax
    rng = np.random.default_rng(7)
    b, k, v = 6, 4, 97
    lp = rng.standard_normal((b, k + 1, v)).astype(np.float32)
    t = lp.argmax(-1).astype(np.int32)
    spec = rng.integers(0, v, (b, k + 1)).astype(np.int32)
    for i in range(b):
        acc = min(i, k)  # row i accepts i draft tokens (row 5: all)
        spec[i, 1 : acc + 1] = t[i, :acc]
        if acc < k:
            spec[i, acc + 1] = (t[i, acc] + 1) % v
    cases.append(("accept_ladder", lp, spec))
    # exact ties: the first maximal index must win
    lp = np.zeros((2, 5, 16), np.float32)
    lp[0, :, 3] = 1.0
    lp[0, :, 9] = 1.0
    lp[1, :, 15] = 2.0
    lp[1, :, 0] = 2.0
    spec = np.array([[0, 3, 3, 3, 3], [1, 0, 0, 15, 0]], np.int32)
    cases.append(("ties_first_index", lp, spec))
    # k = 1 and large-ish vocab
    rng = np.random.default_rng(11)
    lp = (3.0 * rng.standard_normal((3, 2, 4099))).astype(np.float32)
    spec = rng.integers(0, 4099, (3, 2)).astype(np.int32)
    spec[1, 1] = lp[1, 0].argmax()
    cases.append(("k1_v4099", lp, spec))
    return cases


def make_verify(ref: Path) -> None:
    import torch

    mod = _load("ref_verify_torch", ref / "reference" / "cuda_ssd" / "verify_torch.py")
    out = {}
    for name, lp, spec in greedy_cases():
        acc, rec = mod.verify_greedy_torch(torch.tensor(lp), torch.tensor(spec))
        out[f"{name}__logits"] = lp
        out[f"{name}__spec"] = spec
        out[f"{name}__accept_until"] = acc.numpy().astype(np.int32)
        out[f"{name}__recovery"] = rec.numpy().astype(np.int32)
    np.savez_compressed(HERE / "verify_greedy.npz", **out)


def _load_page_manager(ref: Path):
    for pkg in ("jax_ssd", "jax_ssd.runtime"):
        m = types.ModuleType(pkg)
        m.__path__ = []
        sys.modules[pkg] = m
    seq_mod = _load("jax_ssd.runtime.sequence", ref / "jax_ssd" / "runtime" / "sequence.py")
    pm_mod = _load("jax_ssd.runtime.page_manager", ref / "jax_ssd" / "runtime" / "page_manager.py")
    return pm_mod.PageManager, seq_mod.Sequence


def _snap(pm, seqs):
    return {
        "free_blocks": list(pm.free_blocks),
        "ref_counts": {str(k): v for k, v in sorted(pm.ref_counts.items())},
        "block_tables": [list(s.block_table) for s in seqs],
        "draft_block_tables": [list(s.draft_block_table) for s in seqs],
        "num_tokens": [s.num_tokens for s in seqs],
    }


def make_page_manager(ref: Path) -> None:
    PageManager, Sequence = _load_page_manager(ref)
    scenarios = []

    # tests/test_page_rollback.py:5-11
    pm = PageManager(block_size=16, num_blocks=10)
    seq = Sequence(seq_id=0, prompt_token_ids=list(range(20)))
    ops = []
    ok = pm.allocate(seq, 32)
    ops.append({"op": "allocate", "seq": 0, "num_tokens": 32, "ret": ok, "after": _snap(pm, [seq])})
    pm.rollback_speculative(seq, accepted_tokens=4, reserved=20)
    ops.append({"op": "rollback", "seq": 0, "accepted": 4, "reserved": 20, "after": _snap(pm, [seq])})
    scenarios.append({"name": "ref_test_page_rollback", "block_size": 16, "num_blocks": 10,
                      "prompts": [20], "ops": ops})

    # a seeded multi-sequence trace: allocate, draft-allocate, append, rollback, free
    rng = np.random.default_rng(2024)
    for trial in range(6):
        bs = int(rng.choice([4, 16]))
        nb = int(rng.integers(24, 80))
        nseq = int(rng.integers(2, 6))
        pm = PageManager(block_size=bs, num_blocks=nb)
        seqs = [Sequence(seq_id=i, prompt_token_ids=list(range(int(rng.integers(1, 40)))))
                for i in range(nseq)]
        ops = []
        for step in range(40):
            i = int(rng.integers(0, nseq))
            s = seqs[i]
            r = rng.random()
            if r < 0.35:
                n = int(rng.integers(1, 3 * bs))
                ok = pm.allocate(s, n)
                ops.append({"op": "allocate", "seq": i, "num_tokens": n, "ret": ok})
            elif r < 0.45:
                n = int(rng.integers(1, 2 * bs))
                ok = pm.allocate_draft(s, n)
                ops.append({"op": "allocate_draft", "seq": i, "num_tokens": n, "ret": ok})
            elif r < 0.6:
                n = int(rng.integers(1, 6))
                s.append_tokens(list(range(n)))
                ops.append({"op": "append", "seq": i, "n": n})
            elif r < 0.92:
                acc = int(rng.integers(0, 6))
                res = int(rng.integers(0, 3 * bs))
                pm.rollback_speculative(s, accepted_tokens=acc, reserved=res)
                ops.append({"op": "rollback", "seq": i, "accepted": acc, "reserved": res})
            else:
                pm.free_sequence(s)
                ops.append({"op": "free", "seq": i})
            ops[-1]["after"] = _snap(pm, seqs)
        scenarios.append({"name": f"trace_{trial}", "block_size": bs, "num_blocks": nb,
                          "prompts": [len(s.prompt_token_ids) for s in seqs], "ops": ops})

    # shared blocks (ref count 2): the second release returns the block
    pm = PageManager(block_size=4, num_blocks=12)
    a = Sequence(seq_id=0, prompt_token_ids=list(range(6)))
    b = Sequence(seq_id=1, prompt_token_ids=list(range(6)))
    ops = []
    pm.allocate(a, 6)
    ops.append({"op": "allocate", "seq": 0, "num_tokens": 6, "ret": True, "after": _snap(pm, [a, b])})
    b.block_table.extend(a.block_table)  # fork: b shares all of a's blocks
    for blk in a.block_table:
        pm.ref_counts[blk] += 1
    ops.append({"op": "share", "src": 0, "dst": 1, "after": _snap(pm, [a, b])})
    pm.rollback_speculative(a, accepted_tokens=0, reserved=6)
    ops.append({"op": "rollback", "seq": 0, "accepted": 0, "reserved": 6, "after": _snap(pm, [a, b])})
    pm.rollback_speculative(b, accepted_tokens=1, reserved=6)
    ops.append({"op": "rollback", "seq": 1, "accepted": 1, "reserved": 6, "after": _snap(pm, [a, b])})
    scenarios.append({"name": "shared_blocks", "block_size": 4, "num_blocks": 12,
                      "prompts": [6, 6], "ops": ops})

    (HERE / "page_manager.json").write_text(json.dumps(scenarios, indent=None, separators=(",", ":")))


SPEC_CACHE_CASES = {
    # tests/test_spec_cache.py:6-20 (known answers, transcribed)
    "ref_hit_and_miss": {
        "num_branches": 8, "k": 4, "vocab": 32,
        "inserts": [{"slot": 0, "key": [1, 2, 10], "tokens": [5, 6, 7, 8]}],
        "lookups": [{"key": [1, 2, 10], "hit": True, "idx": 0, "tokens": [5, 6, 7, 8]},
                    {"key": [9, 9, 9], "hit": False, "idx": -1, "tokens": [0, 0, 0, 0]}],
    },
}


TOY_CASES = [(64, 32, 0), (100, 32, 3), (64, 16, 7)]  # (vocab_size, hidden_dim, seed)


def make_toy(ref: Path) -> None:
    saved = {k: sys.modules.get(k) for k in ("jax", "jax.numpy", "jax_ssd", "jax_ssd.kernels", "jax_ssd.models")}
    jnp = types.ModuleType("jax.numpy")
    jnp.array, jnp.argmax, jnp.stack = np.asarray, np.argmax, np.stack
    jnp.bfloat16 = np.float32  # a default argument of KVCacheState.allocate, never called here
    jax = types.ModuleType("jax")
    jax.numpy, jax.Array = jnp, np.ndarray  # jax.Array only appears in annotations
    sys.modules["jax"], sys.modules["jax.numpy"] = jax, jnp
    for pkg in ("jax_ssd", "jax_ssd.kernels", "jax_ssd.models"):
        m = types.ModuleType(pkg)
        m.__path__ = []
        sys.modules[pkg] = m
    try:
        _load("jax_ssd.kernels.kv_cache", ref / "jax_ssd" / "kernels" / "kv_cache.py")
        _load("jax_ssd.models.base", ref / "jax_ssd" / "models" / "base.py")
        toy = _load("jax_ssd.models.toy_model", ref / "jax_ssd" / "models" / "toy_model.py")
        out = {}
        for vocab, hidden, seed in TOY_CASES:
            ad = toy.ToyModelAdapter(vocab_size=vocab, hidden_dim=hidden, seed=seed)
            rng = np.random.default_rng(seed + 11)
            ids = np.concatenate([np.arange(2 * hidden), rng.integers(0, 10 * vocab, 40)]).astype(np.int32)
            name = f"v{vocab}_h{hidden}_s{seed}"
            out[f"{name}__ids"] = ids
            out[f"{name}__logits"] = np.asarray(ad.verify(ids, None, None, None).logits, dtype=np.float32)[0]
            prefix = [int(t) for t in ids[:7]]
            spec, lg = ad.draft_speculate(prefix, 5)
            out[f"{name}__draft_prefix"] = np.asarray(prefix, dtype=np.int32)
            out[f"{name}__draft_spec"] = np.asarray(spec, dtype=np.int32)
            out[f"{name}__draft_logits"] = np.asarray(lg, dtype=np.float32)
        np.savez_compressed(HERE / "toy_model.npz", **out)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    make_verify(ref)
    make_page_manager(ref)
    make_toy(ref)
    (HERE / "spec_cache.json").write_text(json.dumps(SPEC_CACHE_CASES, indent=1))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
