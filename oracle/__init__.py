"""ORACLE -- test infrastructure only (never imported by the product).

CPU restatement of the reference kernel's arithmetic (see gemm_oracle.c for
the line-by-line correspondence with src/gemm_kernels.cuh:6-83), a numpy
restatement of the same loop for small cases, and a loader for the reference
kernel itself compiled from source (ref_bank.cu -> _ref/libref_gemm.so) that
the GPU tests use to pin the oracle.
"""
from .gemm_oracle import (  # noqa: F401
    ORACLE_DIR,
    build,
    f16_to_f32,
    f32_to_f16,
    ACTIVATIONS,
    gemm_ex,
    gemm_f16,
    gemm_f16_numpy,
    load,
    load_ref,
    ref_cfgs,
    tolerance,
)
