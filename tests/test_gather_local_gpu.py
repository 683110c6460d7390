"""The fused all-gather's epilogue on one GPU.

gemm_launch_gather stores every finished box of C into each "peer" copy as
well.  Across GPUs those are other GPUs' buffers mapped over NVLink; the
store path does not depend on where the target lives, so here the copies are
buffers on the same GPU.  Each copy must equal C bit for bit, with a
TMA-addressable pitch (one TMA store per copy from the staged box) and with
an odd pitch (16-byte stores from the epilogue warps), and nothing may be
written outside the copies' views."""
import ctypes

import pytest
import torch

import oracle
from helpers import assert_close, make_inputs

pytestmark = pytest.mark.gpu


def _gather(Ad, Bd, M, N, K, cid, ldc, n_copies):
    from infinite_dreams import _capi
    lib = _capi.lib
    big = [torch.full((M + 2, ldc + 3), float("nan"), dtype=torch.float16, device="cuda") for _ in range(n_copies + 1)]
    C = big[0].view(-1)[: M * ldc].view(M, ldc)
    peers = [b.view(-1)[: M * ldc].view(M, ldc) for b in big[1:]]
    arr = (ctypes.c_void_p * max(n_copies, 1))(*[p.data_ptr() for p in peers])
    need = int(lib.gemm_workspace_bytes(Ad.data_ptr(), Bd.data_ptr(), M, N, K, K, N, cid))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    st = lib.gemm_launch_gather(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K, K, N, ldc, arr, n_copies, cid,
                                ws.data_ptr() if need else None, need,
                                torch.cuda.current_stream().cuda_stream or None)
    _capi.check(st, "gemm_launch_gather")
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    _capi.check(lib.gemm_device_error(0, ctypes.byref(code)), "gemm_device_error")
    return C[:, :N], [p[:, :N] for p in peers], C, peers


@pytest.mark.parametrize("knobs", [(256, 256, 64, 6, 2, 1, 2, 1), (256, 512, 64, 4, 2, 1, 8, 1),
                                   (128, 128, 64, 4, 1, 0, 8, 1)])
@pytest.mark.parametrize("pitch_pad", [0, 1])
def test_gather_copies_equal_c(cuda_device, knobs, pitch_pad):
    from infinite_dreams import _capi
    cid = _capi.cfg_find(knobs)
    assert cid >= 0
    M, N, K = 1000, 1536, 640           # ragged M; pitch N (TMA) or N + 1 (per-thread stores)
    A, B = make_inputs(M, N, K, seed=11)
    Ad, Bd = A.cuda(), B.cuda()
    ldc = N + pitch_pad
    C, copies, Cfull, pfull = _gather(Ad, Bd, M, N, K, cid, ldc, 7)
    assert_close(C, oracle.gemm_f16(A.numpy(), B.numpy()), K, f"C {knobs} pitch {ldc}")
    for i, c in enumerate(copies):
        assert torch.equal(c.view(torch.int16), C.view(torch.int16)), f"copy {i} differs ({knobs}, pitch {ldc})"
    if pitch_pad:
        for i, c in enumerate([Cfull] + pfull):
            assert torch.isnan(c[:, N:].float()).all(), f"buffer {i} written outside its view"
