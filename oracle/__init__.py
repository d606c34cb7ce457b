"""CPU oracle for the Bolt-3 hot path.

TEST INFRASTRUCTURE ONLY. This package restates, in plain PyTorch CPU code, the algorithm of the
reference `vsa_lm/config/bolt3.py` (Bolt3Attn forward, _consolidate_functional, Bolt3Decoder.step)
so that the CUDA product can be checked against it. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it, and only as the checker or as
the timed CPU baseline. Nothing in `vsa_lm_b200/` imports it: the product has no CPU fallback.

Parity pin: `tests/golden/make_golden.py` runs the real reference module (imported from its source
tree, which exists only in the build container) on seeded inputs and commits the outputs; the CPU
test `tests/test_oracle_golden.py` checks this oracle against those fixtures.
"""
from .bolt3_oracle import *  # noqa: F401,F403
from .model_oracle import ModelDecoderOracle  # noqa: F401
