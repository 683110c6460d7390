"""GPU parity of the skinny kernel (tile_m = 16 / 32 / 64: C^T tiles, split-K in a cluster).

Each case runs through the C ABI (gemm_launch / gemm_launch_ex) and is
compared with the oracle under |err| <= 1e-2*sqrt(K/1024)*max|C_ref| + 1e-3;
C is poisoned with NaN first, so an unwritten element fails.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, capi_gemm, make_inputs

pytestmark = pytest.mark.gpu


def _cfg(tm, stages, split, tn=128):
    from infinite_dreams import _capi
    cid = _capi.cfg_find((tm, tn, 64, stages, 1, 0, 1, split))
    assert cid >= 0, (tm, tn, stages, split)
    return cid


def _ex(A_st, B_st, M, N, K, tb, cid, alpha=1.0, beta=0.0, D=None, bias=None, act=0, C=None, ta=0):
    from infinite_dreams import _capi
    lib = _capi.lib
    if C is None:
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    lda, ldb = A_st.stride(0), B_st.stride(0)
    need = int(lib.gemm_workspace_bytes_ex(A_st.data_ptr(), B_st.data_ptr(), M, N, K, lda, ldb, ta, tb, cid))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    st = lib.gemm_launch_ex(A_st.data_ptr(), B_st.data_ptr(), C.data_ptr(), M, N, K, lda, ldb, C.stride(0), ta, tb,
                            alpha, beta, D.data_ptr() if D is not None else None, D.stride(0) if D is not None else 0,
                            bias.data_ptr() if bias is not None else None, act, cid,
                            ws.data_ptr() if need else None, need, torch.cuda.current_stream().cuda_stream or None)
    _capi.check(st, "gemm_launch_ex")
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    _capi.check(lib.gemm_device_error(0, ctypes.byref(code)), "gemm_device_error")
    return C


from infinite_dreams import gen_gemm_bank as _gen  # noqa: E402

VARIANTS = _gen.skinny_variants(_gen.enumerate_menu())   # (tile_m, tile_n, stages)


@pytest.mark.parametrize("tm,tn,stages", VARIANTS)
@pytest.mark.parametrize("split", [1, 2, 4, 8])
def test_every_skinny_variant(cuda_device, tm, tn, stages, split):
    """Ragged M (one block and several), N (partial column block) and K (partial 64 block)."""
    for M in (tm - 3, 2 * tm + 5):
        N, K = 1000, 1000
        A, B = make_inputs(M, N, K, dist="skinny", seed=tm + tn + stages + split + M)
        assert_close(capi_gemm(A.cuda(), B.cuda(), _cfg(tm, stages, split, tn)),
                     oracle.gemm_f16(A.numpy(), B.numpy()), K, f"tm {tm} tn {tn} st {stages} S {split} M {M}")


@pytest.mark.parametrize("K", [1, 64, 65, 200, 4096])
def test_cluster_size_clamped_to_k_blocks(cuda_device, K):
    """S = 8 with fewer than 8 K blocks is lowered to a power of two that keeps every CTA busy."""
    M, N = 16, 640
    A, B = make_inputs(M, N, K, seed=K)
    assert_close(capi_gemm(A.cuda(), B.cuda(), _cfg(16, 8, 8)), oracle.gemm_f16(A.numpy(), B.numpy()), K, f"K={K}")


@pytest.mark.parametrize("M", [1, 16, 64])
@pytest.mark.parametrize("N", [4096, 14336])
def test_skinny_workload_shapes_default_cfg(cuda_device, M, N):
    from infinite_dreams import _capi
    K = 4096
    cid = int(_capi.lib.gemm_default_cfg(M, N, K))
    assert _capi.menu_row(cid)[0] < 128
    A, B = make_inputs(M, N, K, dist="skinny", seed=M + N)
    assert_close(capi_gemm(A.cuda(), B.cuda(), cid), oracle.gemm_f16(A.numpy(), B.numpy()), K, f"{M}x{N}x{K}")


@pytest.mark.parametrize("split,tn", [(1, 128), (4, 128), (2, 256)])
def test_skinny_b_stored_n_by_k_and_epilogue(cuda_device, split, tn):
    """y = act(alpha * x @ W.t() + beta * D + b), W stored N x K (K-major B tiles)."""
    M, N, K = 24, 1500, 2048
    g = torch.Generator().manual_seed(split)
    x = (torch.rand((M, K), generator=g) * 2 - 1).half()
    W = (torch.rand((N, K), generator=g) * 0.1 - 0.05).half()
    b = (torch.rand((N,), generator=g) - 0.5).half()
    D = (torch.rand((M, N), generator=g) * 2 - 1).half()
    cid = _cfg(32, 8 if tn == 128 else 6, split, tn)
    plain = _ex(x.cuda(), W.cuda(), M, N, K, 1, cid)
    assert_close(plain, oracle.gemm_ex(x.numpy(), W.numpy(), trans_b=True), K, "W stored N x K")
    for act, name in ((0, "none"), (1, "relu"), (2, "gelu")):
        got = _ex(x.cuda(), W.cuda(), M, N, K, 1, cid, alpha=0.75, beta=-0.5, D=D.cuda(), bias=b.cuda(), act=act)
        ref = oracle.gemm_ex(x.numpy(), W.numpy(), trans_b=True, alpha=0.75, beta=-0.5, D=D.numpy(), bias=b.numpy(),
                             activation=name)
        assert_close(got, ref, K, f"epilogue {name}")


def test_skinny_pitches_and_odd_c(cuda_device):
    """Unaligned A/B pitches (repacked) and a C view whose pitch rules out vector stores."""
    M, N, K = 10, 777, 333
    A, B = make_inputs(M, N, K, seed=3)
    ref = oracle.gemm_f16(A.numpy(), B.numpy())
    Aw = torch.zeros((M, K + 3), dtype=torch.float16, device="cuda")
    Aw[:, :K] = A.cuda()
    Bw = torch.zeros((K, N + 5), dtype=torch.float16, device="cuda")
    Bw[:, :N] = B.cuda()
    Cw = torch.full((M, N + 1), float("nan"), dtype=torch.float16, device="cuda")
    capi_gemm(Aw[:, :K], Bw[:, :N], _cfg(16, 12, 2), C=Cw[:, :N], lda=K + 3, ldb=N + 5, ldc=N + 1, M=M, N=N, K=K)
    assert_close(Cw[:, :N], ref, K, "pitched skinny")
    assert torch.isnan(Cw[:, N:].float()).all(), "wrote outside the C view"


def test_skinny_rejects_a_stored_transposed(cuda_device):
    from infinite_dreams import _capi
    A = torch.zeros((64, 16), dtype=torch.float16, device="cuda")   # K x M storage
    B = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    C = torch.zeros((16, 256), dtype=torch.float16, device="cuda")
    st = _capi.lib.gemm_launch_ex(A.data_ptr(), B.data_ptr(), C.data_ptr(), 16, 256, 64, 16, 256, 256, 1, 0, 1.0,
                                  0.0, None, 0, None, 0, _cfg(16, 8, 1), None, 0, None)
    assert st == _capi.GEMM_ERR_UNSUPPORTED and "trans_a" in _capi.lib.gemm_last_error().decode()


def test_skinny_deterministic(cuda_device):
    """Cluster reduction sums the K slices in rank order: repeated launches give the same bits."""
    M, N, K = 16, 4096, 4096
    A, B = make_inputs(M, N, K, dist="skinny", seed=1)
    Ad, Bd = A.cuda(), B.cuda()
    cid = _cfg(16, 12, 8)
    first = capi_gemm(Ad, Bd, cid)
    for _ in range(3):
        assert torch.equal(capi_gemm(Ad, Bd, cid).view(torch.int16), first.view(torch.int16))


@pytest.mark.parametrize("tm,tn,stages,split", [(16, 128, 12, 1), (64, 128, 8, 1), (16, 512, 3, 1),
                                                (16, 256, 6, 2), (32, 128, 8, 4), (16, 128, 12, 8)])
def test_skinny_tma_store_matches_plain_stores(cuda_device, tm, tn, stages, split):
    """A C whose base and pitch TMA can address takes TMA stores of the staged block; an odd pitch takes
    per-thread stores.  Both give the oracle's result bit for bit, and neither writes outside its view
    (ragged M and N: the TMA clips at the tensor map's extent)."""
    M, N, K = tm + 5, 1000, 700
    A, B = make_inputs(M, N, K, dist="skinny", seed=tm * tn + split)
    ref = oracle.gemm_f16(A.numpy(), B.numpy())
    Ad, Bd = A.cuda(), B.cuda()
    cid = _cfg(tm, stages, split, tn)
    big = torch.full((M + 3, N + 8), float("nan"), dtype=torch.float16, device="cuda")      # pitch 1008: TMA
    capi_gemm(Ad, Bd, cid, C=big[:M, :N], ldc=N + 8, M=M, N=N, K=K)
    odd = torch.full((M + 3, N + 1), float("nan"), dtype=torch.float16, device="cuda")      # pitch 1001: plain
    capi_gemm(Ad, Bd, cid, C=odd[:M, :N], ldc=N + 1, M=M, N=N, K=K)
    assert_close(big[:M, :N], ref, K, f"TMA-stored C tm {tm} tn {tn} S {split}")
    assert torch.equal(big[:M, :N].view(torch.int16), odd[:M, :N].view(torch.int16)), "C paths differ"
    assert torch.isnan(big[:M, N:].float()).all() and torch.isnan(big[M:].float()).all(), "TMA wrote outside C"
    assert torch.isnan(odd[:M, N:].float()).all() and torch.isnan(odd[M:].float()).all(), "wrote outside C"


@pytest.mark.parametrize("split,tn,stages", [(1, 128, 8), (2, 256, 5), (4, 128, 8)])
def test_skinny_epilogue_tma_store_matches_plain_stores(cuda_device, split, tn, stages):
    """The fused epilogue on a TMA-addressable C (pitch a multiple of 8: the staged block goes out by TMA
    stores) against the same epilogue on an odd pitch (per-thread stores): bit for bit, for clusters of
    1, 2 and 4, including an in-place update (D is C).  Both match the oracle."""
    M, N, K = 40, 1536, 2048
    g = torch.Generator().manual_seed(100 + split)
    x = (torch.rand((M, K), generator=g) * 2 - 1).half()
    W = (torch.rand((N, K), generator=g) * 0.1 - 0.05).half()
    b = (torch.rand((N,), generator=g) - 0.5).half()
    D = (torch.rand((M, N), generator=g) * 2 - 1).half()
    cid = _cfg(64, stages, split, tn)
    xd, Wd = x.cuda(), W.cuda()
    for act, name in ((0, "none"), (2, "gelu")):
        ref = oracle.gemm_ex(x.numpy(), W.numpy(), trans_b=True, alpha=0.75, beta=-0.5, D=D.numpy(), bias=b.numpy(),
                             activation=name)
        tma_c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")           # pitch 1536: TMA
        _ex(xd, Wd, M, N, K, 1, cid, alpha=0.75, beta=-0.5, D=D.cuda(), bias=b.cuda(), act=act, C=tma_c)
        odd = torch.full((M, N + 1), float("nan"), dtype=torch.float16, device="cuda")         # pitch 1537: plain
        _ex(xd, Wd, M, N, K, 1, cid, alpha=0.75, beta=-0.5, D=D.cuda(), bias=b.cuda(), act=act, C=odd[:, :N])
        assert_close(tma_c, ref, K, f"TMA-stored epilogue {name} S {split}")
        assert torch.equal(tma_c.view(torch.int16), odd[:, :N].view(torch.int16)), f"C paths differ ({name})"
        assert torch.isnan(odd[:, N:].float()).all(), "wrote outside the C view"
        # in place: C starts as D and is overwritten with act(alpha * acc + beta * C + b)
        inplace = D.cuda().clone()
        _ex(xd, Wd, M, N, K, 1, cid, alpha=0.75, beta=-0.5, D=inplace, bias=b.cuda(), act=act, C=inplace)
        assert torch.equal(inplace.view(torch.int16), tma_c.view(torch.int16)), f"in-place update differs ({name})"
