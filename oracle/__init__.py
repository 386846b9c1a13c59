"""Test infrastructure: a CPU restatement of the reference's hot path, used only as the checker.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package. The
product (the package next to it) never does: it runs the CUDA kernels or fails.

Parity is pinned: tests/golden/ holds vectors made by running the reference itself
(qwen38_inf2, imported from the reference checkout by tests/golden/make_golden.py), and
tests/test_oracle_golden.py checks this restatement against them.
"""
