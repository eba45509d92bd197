"""CPU oracle for the verify-pass hot path: TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of mlx-tree-spec's verify pass:
the MLX 4-bit affine (group 64) weight format and its quantized matmul, the
tree ancestor masks, tree-mask attention over a long KV prefix, and the 8-bit
KV formats. It is the checker that the CUDA library is compared against, and
the CPU baseline that bench.py times beside it. Nothing in the shipped library
(`mlx-tree-spec_b200/`) imports it: only tests/, __graft_entry__.smoke() and
bench.py's CPU legs do.

Parity status:
  * pinned: the weight format (nibble order, group layout) against the
    reference's kernels and relayout code, and the ancestor bitmask against the
    reference's own known-answer test (tests/test_units.py:29-32);
  * partially pinned: the qmm and attention numerics. The reference's
    arithmetic lives in MLX 0.32.2 / MTPLX 2.12.2 Metal kernels that cannot run
    here (no Metal, packages absent), so outputs are checked against this
    float64 restatement with the tolerance the reference's own test implies
    (max-abs-err <= 2e-2 * max|ref| for bf16 outputs) rather than against MLX
    outputs.
"""

from . import bf16, qmm, tree, attention, kv, gen  # noqa: F401
