"""CPU oracle for the paged-KV execution path — TEST INFRASTRUCTURE, not product code.

This package restates, on the CPU, what the reference computes on the hot path so that the
CUDA kernels can be checked against it:

* ``paged_kv``  — slot mapping, shadow-KV write/verify, pool scatter/gather and block copy
  (tokenserve ``src/tokenserve/backends/base.py:40-45``,
  ``src/tokenserve/backends/simulated.py:147-169``), in numpy integer arithmetic.
* ``attention`` — eager attention with grouped-query heads and a causal mask (transformers
  5.5.0 ``models/llama/modeling_llama.py:187-222``, called by tokenserve
  ``src/tokenserve/backends/hf.py:71``), in numpy float64 for parity and in torch-CPU float32
  for the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import this package, and only as the checker or the timed CPU baseline; the product package
``tokenserve_b200`` never imports it.

Parity pin: the oracle is checked against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports tokenserve and transformers and records their
outputs) and against the reference's own known-answer test for the slot mapping
(``tests/test_simulated_backend.py:77-79``).
"""
