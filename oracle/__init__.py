"""Test-only checker: CPU restatement of the reference kernels and the harness
around the reference's own kernels.  Imported only by tests/, the smoke test
and the CPU-baseline legs of bench.py."""

from .oracle import (  # noqa: F401
    Oracle,
    REF_LIB,
    REF_LIB_PTX,
    RefKernels,
    bf16_to_f32,
    bf16_ulp,
    f32_to_bf16,
    ulp_error,
)
