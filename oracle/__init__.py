"""CPU oracle for the fused forward-Laplacian hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may use
it, and only as the checker (or the timed CPU baseline), never as the product path.

Two independent restatements of the reference algorithm live here:

* :mod:`oracle.jet` -- PyTorch on the CPU, restating the reference's own PyTorch oracle
  (``src/fused_hoad/backends/forward_laplacian.py``, ``src/fused_hoad/autodiff.py``,
  ``src/fused_hoad/backends/fused.py:_recompute_backward``). PyTorch is the reference's
  only arithmetic dependency (``pyproject.toml:13``), so the same matmul/tanh arithmetic
  defines parity.
* :mod:`oracle.cjet` -- a plain-C FP64 restatement of the forward jet and of the
  hand-derived adjoint-jet backward (the closed forms of ``csrc/fused_backward.cu:29-33``
  and ``:75-89``), built by :mod:`oracle.build` into ``oracle/_build/``.

Parity is pinned: ``tests/golden/make_golden.py`` imports the unmodified reference package
and records its outputs into ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks
both restatements against those vectors.
"""
