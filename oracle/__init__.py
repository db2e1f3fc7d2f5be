"""CPU oracle for the Fry int8 forward pass. TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU with torch, what the reference
(GilliamWong/chess-transformer) computes on the path this repository
accelerates: the batched int8 forward of Fry's network over encoded leaf
positions. Every function cites the reference file:line it follows.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline /
reference arm may import it, and only as the checker or as the timed CPU
baseline. The product path (`chess-transformer_b200/`) never imports it and
has no CPU fallback.

Pinning: `tests/golden/make_golden.py` imports the reference's own
`model/model.py`, `model/fused_blocks.py`, `model/int8_blocks.py` and
`engine/quantization.py` (python-chess replaced by a stub that rebuilds the
move table) and runs the reference's Triton kernels under the Triton
interpreter; the fixtures it writes under `tests/golden/` are what
`tests/test_oracle_golden.py` checks this package against.
"""
