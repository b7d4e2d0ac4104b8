"""CPU oracle for the W8A8 hot path: TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's own CPU references (AshrithaG/int8-linear):
the exact int32 product and float64 scaled layer of tests/test_kernel.py and
bench/bench_linear.py, and the quantiser references of tests/test_fused_quant.py.
Each function cites the reference file:line it restates.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU baseline.  The
product path (the int8_linear package) never imports it; with the CUDA library
missing the product raises instead of falling back to anything here.

Pinned by tests/golden/ (fixtures made by tests/golden/make_golden.py, which runs the
reference's own functions on seeded CPU inputs) through tests/test_oracle_golden.py.
"""
