"""Test helpers: seeded inputs, the C-ABI call path and the parity check."""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np
import torch

import oracle


def make_inputs(M: int, N: int, K: int, dist: str = "uniform", seed: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded CPU fp16 inputs (fp32 draw -> fp16), as the workloads specify."""
    g = torch.Generator().manual_seed(seed)
    if dist == "uniform":
        A = torch.rand((M, K), generator=g, dtype=torch.float32) * 2 - 1
        B = torch.rand((K, N), generator=g, dtype=torch.float32) * 2 - 1
    elif dist == "skinny":
        A = torch.randn((M, K), generator=g, dtype=torch.float32)
        B = torch.randn((K, N), generator=g, dtype=torch.float32) * 0.02
    else:
        raise ValueError(dist)
    return A.to(torch.float16), B.to(torch.float16)


def capi_gemm(A: torch.Tensor, B: torch.Tensor, cfg_id: int, C: Optional[torch.Tensor] = None,
              lda: Optional[int] = None, ldb: Optional[int] = None, ldc: Optional[int] = None,
              M: Optional[int] = None, N: Optional[int] = None, K: Optional[int] = None) -> torch.Tensor:
    """C = A*B through gemm_launch of the C ABI (device tensors, explicit workspace)."""
    from infinite_dreams import _capi
    lib = _capi.lib
    M = A.shape[0] if M is None else M
    K = A.shape[1] if K is None else K
    N = B.shape[1] if N is None else N
    lda = A.stride(0) if lda is None else lda
    ldb = B.stride(0) if ldb is None else ldb
    if C is None:
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device=A.device)
    ldc = C.stride(0) if ldc is None else ldc
    need = int(lib.gemm_workspace_bytes(A.data_ptr(), B.data_ptr(), M, N, K, lda, ldb, cfg_id))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=A.device)
    stream = torch.cuda.current_stream(A.device).cuda_stream
    st = lib.gemm_launch(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, lda, ldb, ldc, cfg_id,
                         ws.data_ptr() if need else None, need, stream or None)
    _capi.check(st, "gemm_launch")
    torch.cuda.synchronize(A.device)
    code = ctypes.c_int(0)
    _capi.check(lib.gemm_device_error(A.device.index or 0, ctypes.byref(code)), "gemm_device_error")
    if need:
        # every successful launch leaves the ticket region zero
        cnt = int(lib.gemm_workspace_counter_bytes())
        assert int(ws[:cnt].count_nonzero()) == 0, "split-K tickets not reset"
    return C


def oracle_gemm(A: torch.Tensor, B: torch.Tensor) -> np.ndarray:
    return oracle.gemm_f16(A.cpu().numpy(), B.cpu().numpy())


def assert_close(C: torch.Tensor, ref: np.ndarray, K: int, what: str = "") -> float:
    """|C - ref| <= 1e-2*sqrt(K/1024)*max|ref| + 1e-3 elementwise; returns max error."""
    got = C.detach().float().cpu().numpy()
    exp = np.asarray(ref, dtype=np.float32)
    assert got.shape == exp.shape, (got.shape, exp.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output (unwritten tile?)"
    err = float(np.max(np.abs(got - exp))) if got.size else 0.0
    tol = oracle.tolerance(exp, K)
    assert err <= tol, f"{what}: max|err| {err} > tol {tol}"
    return err
