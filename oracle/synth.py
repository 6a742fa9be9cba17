"""Seeded synthetic inputs for the oracle and the tests (TEST INFRASTRUCTURE).

The generator itself lives in fftsparse_b200/synthetic.py so that bench.py can
build its workload without importing anything under oracle/; this module only
re-exports it for the checkers.
"""
from fftsparse_b200.synthetic import apply_rope, expand_kv, make_inputs, rope_cos_sin  # noqa: F401
