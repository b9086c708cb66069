"""CPU oracle of the reference's tile programs -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU baseline / reference arm, and only as
the checker or the timed CPU baseline.  The product path (pytorchsim-triton-backend_b200/) never imports it.
Parity is pinned: tests/test_oracle_golden.py checks these restatements against output vectors of the
reference's own Triton kernels (tests/golden/make_golden.py runs them under the Triton interpreter)."""
