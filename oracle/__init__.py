"""CPU oracle for the fused FP8 block-scale MoE hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (``flashinfer_b200``) imports this package. Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
legs of ``bench.py`` use it, and only as the checker or the timed CPU baseline.

It restates, in numpy, the reference's algorithm for the path:

* routing: ``solution/triton/kernel.py:371-457`` (``_route_select_local_kernel``)
  and the operator definition's PyTorch reference
  ``flashinfer/trace/templates/moe.py:109-184``
  (flashinfer-python 0.6.11.post2, the in-container copy of the definition);
* permutation: ``kernel.py:519-597`` with the canonical order of
  ``moe.py:79-98`` (local experts ascending, tokens ascending within each);
* expert compute: ``moe.py:28-100`` (fp32 dequantise, loop over experts,
  SwiGLU = silu(second half) * first half, weighted ``index_add_``, bf16 cast).

Parity pin: ``tests/test_oracle_pins.py`` checks these functions against the
golden vectors in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by running the installed definition reference itself.
"""
