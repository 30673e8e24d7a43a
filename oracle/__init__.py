"""CPU oracle for the quantized GEMM hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``bench.py``'s CPU-baseline leg and
``__graft_entry__.smoke()`` may import this package, and only as the checker.
The product (``hotarubi_b200`` and ``libhrb_gemm.so``) never imports it.

Two checkers live here:

* ``_build/libhrb_oracle.so``: the C restatement in ``hrb_oracle.c`` (pinned
  against the reference below and against ``tests/golden/``);
* ``_ref/libhrb_ref.so``: hotarubi's own GEMM sources compiled where they lie
  in the reference checkout (``Makefile`` target ``ref``), present wherever it
  was built (it is shipped with the repository snapshot, not committed).
"""
