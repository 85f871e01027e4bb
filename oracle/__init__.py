"""CPU oracle for the pdum_dsl_b200 hot path -- TEST INFRASTRUCTURE ONLY.

A numpy float64 restatement of the reference evaluator's results on the
attention and row-reduction regions (pdum.tl.dialect.run_region,
packages/tensorlib/src/pdum/tl/dialect.py:1349-1473, over the naive regions
of pdum/tl/zoo/attention.py:167-196 and zoo_common.py:56-86).

Parity pin: tests/test_oracle.py checks these functions against golden
vectors that tests/golden/make_golden.py produced by running the reference's
own run_region on the same seeded inputs (fixtures under tests/golden/).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker or the timed CPU
baseline.  The product path (pdum_dsl_b200) never imports it.
"""
