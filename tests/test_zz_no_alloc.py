"""gemm_launch_noalloc: the launch for callers that cannot allocate device memory.

Some callers get nothing but input/output pointers and a stream: an operator
inside a runtime that plans all device buffers in advance, or a plugin next
to a framework whose allocator already holds almost all of the GPU's memory.
They cannot cudaMalloc a workspace, so this entry point keeps split-K
partials, tickets and repacked operands in a fixed 32 MiB array inside the
library.  These tests call it through the C ABI, twice in a row on problems
that need that scratch, and compare each result with gemm_launch (which is
given a workspace allocated here) under the parity tolerance of the other
GPU tests.  The file sorts last so that a failure here stops a `-x` run only
after every other test has run; it also passes in a fresh process.
"""
import pytest
import torch

from helpers import assert_close, capi_gemm, make_inputs

pytestmark = pytest.mark.gpu


def _cfg(tile_n, stages, split_k):
    from infinite_dreams import _capi
    cid = _capi.cfg_find((128, tile_n, 64, stages, 1, 0, 8, split_k))
    assert cid >= 0
    return cid


def _noalloc(A, B, cfg_id, M, N, K):
    from infinite_dreams import _capi
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device=A.device)
    stream = torch.cuda.current_stream(A.device).cuda_stream
    st = _capi.lib.gemm_launch_noalloc(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, A.stride(0),
                                       B.stride(0), N, cfg_id, stream or None)
    _capi.check(st, "gemm_launch_noalloc")
    torch.cuda.synchronize(A.device)
    return C


# (M, N, K, tile_n, stages, split_k): all need scratch; the third also repacks
# A (K=777 is not a TMA-addressable pitch) on top of split-K partials.
CASES = [
    (64, 4096, 4096, 128, 6, 4),
    (200, 1536, 2048, 128, 4, 8),
    (1000, 3000, 777, 128, 6, 2),
]


def test_noalloc_matches_gemm_launch_two_calls_in_a_row(cuda_device):
    from infinite_dreams import _capi
    for i, (M, N, K, bn, st, sk) in enumerate(CASES):
        cid = _cfg(bn, st, sk)
        need = _capi.lib.gemm_workspace_bytes(1 << 20, 1 << 20, M, N, K, K, N, cid)
        assert 0 < need <= 32 * 1024 * 1024
        A, B = make_inputs(M, N, K, seed=40 + i)
        Ad, Bd = A.cuda(), B.cuda()
        expect = capi_gemm(Ad, Bd, cid)                       # existing entry point, own workspace
        ref = expect.float().cpu().numpy()
        first = _noalloc(Ad, Bd, cid, M, N, K)
        second = _noalloc(Ad, Bd, cid, M, N, K)               # the array keeps the first call's contents
        assert_close(first, ref, K, f"noalloc first call {M}x{N}x{K}")
        assert_close(second, ref, K, f"noalloc second call {M}x{N}x{K}")
        # Same kernels, same K order: a stale partial or ticket left in the
        # shared array by the first call would show up as a bit difference.
        assert torch.equal(first.view(torch.int16), expect.view(torch.int16)), f"first call {M}x{N}x{K}"
        assert torch.equal(second.view(torch.int16), expect.view(torch.int16)), f"second call {M}x{N}x{K}"
    from infinite_dreams import infinite_dreams_ext as ext
    ext.check_device_errors()


def test_noalloc_rejects_problems_above_the_static_scratch(cuda_device):
    from infinite_dreams import _capi
    M, N, K = 128, 14336, 4096
    cid = _cfg(128, 6, 8)      # 112 tiles x 8 splits x 64 KiB of partials > 32 MiB
    assert _capi.lib.gemm_workspace_bytes(1 << 20, 1 << 20, M, N, K, K, N, cid) > 32 * 1024 * 1024
    A = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    B = torch.zeros((K, N), dtype=torch.float16, device="cuda")
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    st = _capi.lib.gemm_launch_noalloc(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N, cid,
                                       torch.cuda.current_stream().cuda_stream or None)
    assert st == _capi.GEMM_ERR_WORKSPACE
    assert "static buffer" in _capi.lib.gemm_last_error().decode()
    torch.cuda.synchronize()
    assert torch.isnan(C.float()).all(), "a rejected call must not launch"
