"""CPU oracle for the paged-KV attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy and plain Python, the reference algorithm of
each operation the sm_100a library replaces. It is the checker the parity
tests compare the CUDA path against, and the timed CPU baseline of bench.py.
Nothing in serving_engine_b200 imports it: the product path has no CPU
fallback and fails loudly when its CUDA library is missing.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline and
--impl reference legs) may import this package.

Pinning: tests/golden/ holds outputs of the reference itself run in this
container (its eager paged-attention path, its Triton kernel under the Triton
interpreter, its index_copy_ KV write and its build_paged_batch_metadata),
made by tests/golden/make_golden.py; tests/test_oracle_golden.py checks every
function here against them.
"""
