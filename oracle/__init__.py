"""CPU oracle for the speculative-decoding verify step — TEST INFRASTRUCTURE ONLY.

This package checks results and is never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The shipped path (``ssd_b200``) runs the CUDA library and fails
loudly when that library is missing; it never routes through this code.

It restates, in numpy, the reference's algorithms for the verify path of
``TinevimboMusingadi/ssd-tpu-`` (a JAX engine whose own code cannot be imported
here: jax is not installed).  Each function cites the reference file:line it
follows.

Pinning status
--------------
* greedy accept/recovery (``verify.verify_greedy``): pinned — checked against
  golden vectors produced by the reference's ``reference/cuda_ssd/verify_torch.py``
  (``tests/golden/verify_greedy.npz``).
* page allocation / rollback / free (``page_manager``): pinned — checked against
  traces produced by running the reference's ``jax_ssd/runtime/page_manager.py``
  (``tests/golden/page_manager.json``).
* spec-cache lookup (``spec_cache``): pinned to the known answers of the
  reference's ``tests/test_spec_cache.py``.
* sampling-mode verify (``verify.verify_sample``), paged attention, KV write
  and the Gemma forward: parity unpinned — restated from the reference source
  (and, for the Gemma arithmetic, from the architecture; cross-checked against
  the torch ``GemmaForCausalLM`` of the installed transformers in fp32), with no
  reference run possible in this container.
"""
