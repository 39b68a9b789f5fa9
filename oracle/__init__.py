"""TEST INFRASTRUCTURE ONLY — CPU oracle for the pytorch_opt.ops hot path.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it. Nothing in ``pytorch_opt_b200`` imports, links or executes it.

* ``oracle.ops_np`` restates, in numpy, the reference algorithms of
  kavinravi/pytorch-opt for this path (each function cites the reference
  file:line it follows).
* Parity is pinned: ``tests/test_oracle_golden.py`` checks every function
  here against golden vectors produced by the reference itself
  (``tests/golden/make_golden.py`` imports the reference package and commits
  its inputs and outputs as ``tests/golden/*.npz``).
* ``oracle/build_ref.py`` compiles the reference's own native ATen source
  (``pytorch_opt/ops/csrc/pytorch_opt_ops.cpp``) with g++ into
  ``oracle/_ref/`` (git-ignored, shipped with the tree); ``oracle.ref_native``
  loads it. It serves as the timed CPU baseline ("reference" kind) and as a
  second cross-check of the restatement.
"""
