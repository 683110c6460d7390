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


def _gather_copy(Ad, Bd, M, N, K, cid, ldc, n_copies, n_streams):
    from infinite_dreams import _capi
    lib = _capi.lib
    big = [torch.full((M + 2, ldc + 3), float("nan"), dtype=torch.float16, device="cuda") for _ in range(n_copies + 1)]
    C = big[0].view(-1)[: M * ldc].view(M, ldc)
    peers = [b.view(-1)[: M * ldc].view(M, ldc) for b in big[1:]]
    arr = (ctypes.c_void_p * max(n_copies, 1))(*[p.data_ptr() for p in peers])
    streams = [torch.cuda.Stream() for _ in range(n_streams)]
    sarr = (ctypes.c_void_p * n_streams)(*[s.cuda_stream for s in streams])
    counters = torch.full((_capi.GEMM_GATHER_COUNTERS,), 12345, dtype=torch.int32, device="cuda")
    need = int(lib.gemm_workspace_bytes(Ad.data_ptr(), Bd.data_ptr(), M, N, K, K, N, cid))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    st = lib.gemm_launch_gather_copy(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K, K, N, ldc, arr, n_copies,
                                     cid, ws.data_ptr() if need else None, need,
                                     torch.cuda.current_stream().cuda_stream or None, sarr, n_streams,
                                     counters.data_ptr())
    _capi.check(st, "gemm_launch_gather_copy")
    # the copy streams were joined into the launch stream: syncing it covers every copy
    torch.cuda.current_stream().synchronize()
    code = ctypes.c_int(0)
    _capi.check(lib.gemm_device_error(0, ctypes.byref(code)), "gemm_device_error")
    return C[:, :N], [p[:, :N] for p in peers], C, peers, counters


@pytest.mark.parametrize("knobs", [(256, 256, 64, 6, 2, 1, 2, 1), (256, 512, 64, 4, 2, 1, 8, 1),
                                   (128, 128, 64, 4, 1, 0, 8, 1)])
@pytest.mark.parametrize("M,N,K,pad", [(2048, 16384, 512, 0), (1000, 1536, 640, 1), (300, 5000, 200, 0)])
def test_gather_copy_engines_copies_equal_c(cuda_device, knobs, M, N, K, pad):
    """Copy-engine exchange: the kernel's chunk walk and counts, the GPU-side waits and the copies (2-D
    column strips and the contiguous tail rows) give every copy C bit for bit; the counts end at one
    signal per epilogue warp per tile; nothing outside the views is written."""
    from infinite_dreams import _capi
    cid = _capi.cfg_find(knobs)
    assert cid >= 0
    A, B = make_inputs(M, N, K, seed=12)
    Ad, Bd = A.cuda(), B.cuda()
    ldc = N + pad
    for n_copies, n_streams in ((7, 14), (3, 3), (1, 1)):
        C, copies, Cfull, pfull, counters = _gather_copy(Ad, Bd, M, N, K, cid, ldc, n_copies, n_streams)
        if n_copies == 7:
            assert_close(C, oracle.gemm_f16(A.numpy(), B.numpy()), K, f"C {knobs} {M}x{N}x{K}")
        for i, c in enumerate(copies):
            assert torch.equal(c.view(torch.int16), C.view(torch.int16)), f"copy {i} differs ({knobs} {M}x{N}x{K})"
        bm, bn, cg = 128 * knobs[4], knobs[1], knobs[4]
        tiles = ((M + bm - 1) // bm) * ((N + bn - 1) // bn)
        assert int(counters.sum()) == tiles * 4 * cg, counters.tolist()
        if pad:
            for i, c in enumerate([Cfull] + pfull):
                assert torch.isnan(c[:, N:].float()).all(), f"buffer {i} written outside its view"


def test_gather_copy_rejects_bad_streams_and_configs(cuda_device):
    from infinite_dreams import _capi
    lib = _capi.lib
    M = N = K = 512
    A = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    B = torch.zeros((K, N), dtype=torch.float16, device="cuda")
    C = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    P = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    arr = (ctypes.c_void_p * 1)(P.data_ptr())
    counters = torch.zeros(_capi.GEMM_GATHER_COUNTERS, dtype=torch.int32, device="cuda")
    cur = torch.cuda.current_stream().cuda_stream
    good = _capi.cfg_find((128, 128, 64, 4, 1, 0, 8, 1))
    split = _capi.cfg_find((128, 128, 64, 4, 1, 0, 8, 2))
    s = torch.cuda.Stream()
    same = (ctypes.c_void_p * 1)(cur) if cur else None
    if same is not None:
        st = lib.gemm_launch_gather_copy(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N, arr, 1, good,
                                         None, 0, cur, same, 1, counters.data_ptr())
        assert st == _capi.GEMM_ERR_INVALID_ARG
    ok = (ctypes.c_void_p * 1)(s.cuda_stream)
    st = lib.gemm_launch_gather_copy(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N, arr, 1, good,
                                     None, 0, cur or None, ok, 1, None)
    assert st == _capi.GEMM_ERR_INVALID_ARG and "chunk_counters" in lib.gemm_last_error().decode()
    if split >= 0:
        ws = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
        st = lib.gemm_launch_gather_copy(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N, arr, 1, split,
                                         ws.data_ptr(), ws.numel(), cur or None, ok, 1, counters.data_ptr())
        assert st == _capi.GEMM_ERR_UNSUPPORTED
    torch.cuda.synchronize()
