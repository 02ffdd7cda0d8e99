"""CPU oracle for the int4 speech-LM decode path (test infrastructure only).

This package restates, on the CPU, the arithmetic of the reference's decode path so
that the CUDA library can be checked against it.  It is imported only by the tests,
by ``__graft_entry__.smoke()`` (as the checker) and by the CPU-baseline leg of
``bench.py``.  The product library never calls into it.

Parity status: the reference (Swift + MLX + Metal) cannot be built or run on this
machine (no Swift toolchain, no MLX, no Apple GPU).  The integer/control-flow parts
(code packing, loop guard, runaway retry, acceptance, KV rollback) are pinned by the
reference's own known-answer tests, restated in ``tests/test_oracle_pins.py``.  The
floating-point parts (product-form dequant GEMM, RMSNorm, RoPE, attention, LayerNorm,
GELU) follow the reference's formulas but are *parity unpinned* against MLX, because
no MLX output vectors exist in the reference repository.
"""
