"""CPU oracle for the RecoverSSM verify + grouped-commit path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this folder.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, always as the checker or the
CPU baseline, never as the thing measured on the GPU.

* ``gdn_oracle``    -- float64 NumPy restatement of the reference algorithm
  (verify recurrence, record layout, commit fold, commit plans, conv
  compaction, align publication), one function per reference kernel, each
  citing the reference file:line it follows.
* ``cpu_executors`` -- torch CPU executors (float32, vectorised over rows and
  heads, all host threads) restating the reference's own CPU executors; used
  as the timed CPU baseline.

Pinning: ``tests/test_oracle_pins.py`` checks this oracle against the
reference's known-answer tests and against fixtures produced by running the
reference's own Triton kernels (``tests/golden/make_golden.py``).
"""
