"""The oracle: C restatement vs numpy restatement vs golden vectors produced
by the reference kernel itself (tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_gemm_golden.npz"


def test_f16_to_f32_exhaustive():
    h = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_to_f32(h)
    exp = h.view(np.float16).astype(np.float32)
    nan = np.isnan(exp)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), exp[~nan].view(np.uint32))


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(1)
    parts = [rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-3, 1.0, 300.0, 6e4)]
    # every half value, and the midpoints between neighbours (ties)
    h = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    mids = ((h[:-1] + h[1:]) / 2).astype(np.float32)
    edge = np.array([65504, 65519.996, 65520, 65536, 1e9, 2.98023224e-08, 5.96e-08, 0.0, -0.0, np.inf, -np.inf],
                    dtype=np.float32)
    x = np.concatenate(parts + [mids, -mids, edge])
    with np.errstate(over="ignore"):
        exp = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16(x), exp)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (7, 13, 29), (64, 96, 200), (5, 300, 777), (130, 70, 65), (3, 4, 0)])
def test_c_oracle_equals_numpy_restatement(M, N, K):
    rng = np.random.default_rng(M * 1000 + N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    for threads in (1, 3, 8):
        c = oracle.gemm_f16(A, B, threads=threads)
        assert np.array_equal(c.view(np.uint16), oracle.gemm_f16_numpy(A, B).view(np.uint16))


def test_oracle_is_close_to_fp32_matmul():
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (64, 512)).astype(np.float16)
    B = rng.uniform(-1, 1, (512, 96)).astype(np.float16)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    got = oracle.gemm_f16(A, B).astype(np.float64)
    assert np.max(np.abs(got - ref)) <= oracle.tolerance(ref, 512)


@pytest.fixture(scope="module")
def golden():
    if not GOLDEN.exists():
        pytest.skip("golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    return np.load(GOLDEN)


def test_oracle_matches_reference_kernel_golden(golden):
    names = list(golden["cases"])
    assert len(names) >= 8
    for name in names:
        A = golden[f"{name}__A"].view(np.float16)
        B = golden[f"{name}__B"].view(np.float16)
        C = golden[f"{name}__C"]
        got = oracle.gemm_f16(A, B).view(np.uint16)
        assert np.array_equal(got, C), name
        assert np.array_equal(oracle.gemm_f16_numpy(A, B).view(np.uint16), C), name


def test_golden_planted_mistake_is_caught(golden):
    """A one-ulp change to one oracle output must be detected."""
    name = list(golden["cases"])[3]
    A = golden[f"{name}__A"].view(np.float16)
    B = golden[f"{name}__B"].view(np.float16)
    got = oracle.gemm_f16(A, B).view(np.uint16).copy()
    got[0, 0] ^= 1
    assert not np.array_equal(got, golden[f"{name}__C"])
