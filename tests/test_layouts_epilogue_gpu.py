"""GPU parity: transposed operand storage and the fused epilogue (gemm_launch_ex).

Every case runs through the C ABI and is compared with ``oracle.gemm_ex``
(the oracle's sequential-k fp32 accumulation with the same transposed reads
and the epilogue act(alpha * acc + beta * D + bias) in fp32, rounded once)
under the acceptance bound |err| <= 1e-2*sqrt(K/1024)*max|C_ref| + 1e-3.
Outputs are poisoned with NaN first, so an unwritten element fails.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, capi_gemm, make_inputs

pytestmark = pytest.mark.gpu

ACT = {"none": 0, "relu": 1, "gelu": 2}


def _cfg(tile_n=128, stages=4, raster=0, group=8, split_k=1, mma_sm=1):
    from infinite_dreams import _capi
    cid = _capi.cfg_find((128 * mma_sm, tile_n, 64, stages, mma_sm, raster, group, split_k))
    assert cid >= 0
    return cid


def _stored(X: torch.Tensor, trans: bool, pad: int = 0) -> torch.Tensor:
    """X ([R, C] logical) as stored on the GPU: itself, or its transpose
    materialised; `pad` extra elements of row pitch (a view into a wider buffer)."""
    S = (X.t().contiguous() if trans else X.contiguous()).cuda()
    if pad:
        W = torch.zeros((S.shape[0], S.shape[1] + pad), dtype=S.dtype, device="cuda")
        W[:, :S.shape[1]] = S
        S = W[:, :S.shape[1]]
    return S


def capi_gemm_ex(A_st, B_st, M, N, K, ta, tb, cfg_id, alpha=1.0, beta=0.0, D=None, bias=None, act="none",
                 C=None):
    """Launch gemm_launch_ex on device tensors A_st / B_st (stored orientation, any pitch)."""
    from infinite_dreams import _capi
    lib = _capi.lib
    lda, ldb = A_st.stride(0), B_st.stride(0)
    if C is None:
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    need = int(lib.gemm_workspace_bytes_ex(A_st.data_ptr(), B_st.data_ptr(), M, N, K, lda, ldb, ta, tb, cfg_id))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    st = lib.gemm_launch_ex(A_st.data_ptr(), B_st.data_ptr(), C.data_ptr(), M, N, K, lda, ldb, C.stride(0), ta, tb,
                            alpha, beta, D.data_ptr() if D is not None else None,
                            D.stride(0) if D is not None else 0, bias.data_ptr() if bias is not None else None,
                            ACT[act], cfg_id, ws.data_ptr() if need else None, need,
                            torch.cuda.current_stream().cuda_stream or None)
    _capi.check(st, "gemm_launch_ex")
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    _capi.check(lib.gemm_device_error(0, ctypes.byref(code)), "gemm_device_error")
    if need:
        assert int(ws[:int(lib.gemm_workspace_counter_bytes())].count_nonzero()) == 0, "tickets not reset"
    return C


def _ref(A, B, ta, tb, **kw):
    A_st = A.t().contiguous() if ta else A
    B_st = B.t().contiguous() if tb else B
    kw = {k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    return oracle.gemm_ex(A_st.numpy(), B_st.numpy(), trans_a=ta, trans_b=tb, **kw)


LAYOUTS = [(0, 0), (1, 0), (0, 1), (1, 1)]
KERNELS = [dict(tile_n=64, stages=5), dict(tile_n=128, stages=4), dict(tile_n=192, stages=4),
           dict(tile_n=256, stages=4), dict(tile_n=128, stages=4, mma_sm=2), dict(tile_n=256, stages=4, mma_sm=2),
           dict(tile_n=512, stages=3, mma_sm=2)]


@pytest.mark.parametrize("ta,tb", LAYOUTS)
@pytest.mark.parametrize("kern", KERNELS, ids=lambda k: f"bn{k['tile_n']}_cg{k.get('mma_sm', 1)}")
def test_layouts_every_kernel(cuda_device, ta, tb, kern):
    """All four storage orders on ragged M/N/K edges; the sum is the same GEMM."""
    M, N, K = 320, 1100, 328
    A, B = make_inputs(M, N, K, seed=7 * ta + 3 * tb + kern["tile_n"])
    ref = oracle.gemm_f16(A.numpy(), B.numpy())
    C = capi_gemm_ex(_stored(A, ta), _stored(B, tb), M, N, K, ta, tb, _cfg(**kern))
    assert_close(C, ref, K, f"layout ({ta},{tb}) {kern}")


@pytest.mark.parametrize("ta,tb", LAYOUTS[1:])
def test_transposed_equals_row_major_bitwise(cuda_device, ta, tb):
    """Same products in the same MMA K order: storage order must not change a bit."""
    M, N, K = 512, 768, 1024
    A, B = make_inputs(M, N, K, seed=21)
    for kern in (dict(tile_n=256, stages=4), dict(tile_n=512, stages=4, mma_sm=2)):
        cid = _cfg(**kern)
        base = capi_gemm(A.cuda(), B.cuda(), cid)
        C = capi_gemm_ex(_stored(A, ta), _stored(B, tb), M, N, K, ta, tb, cid)
        assert torch.equal(base.view(torch.int16), C.view(torch.int16)), f"({ta},{tb}) {kern}"


@pytest.mark.parametrize("ta,tb", LAYOUTS)
@pytest.mark.parametrize("knobs", [dict(split_k=4), dict(split_k=0), dict(tile_n=256, stages=4, split_k=3)])
def test_layouts_split_and_stream_k(cuda_device, ta, tb, knobs):
    M, N, K = 200, 900, 1500
    A, B = make_inputs(M, N, K, dist="skinny", seed=ta + 2 * tb)
    ref = oracle.gemm_f16(A.numpy(), B.numpy())
    C = capi_gemm_ex(_stored(A, ta), _stored(B, tb), M, N, K, ta, tb, _cfg(**knobs))
    assert_close(C, ref, K, f"({ta},{tb}) {knobs}")


@pytest.mark.parametrize("ta,tb", LAYOUTS)
def test_layouts_unaligned_pitches_repack(cuda_device, ta, tb):
    """Stored pitches that TMA cannot address: the operand is repacked in its stored orientation."""
    M, N, K = 150, 333, 203
    A, B = make_inputs(M, N, K, seed=5 + ta + tb)
    ref = oracle.gemm_f16(A.numpy(), B.numpy())
    A_st, B_st = _stored(A, ta, pad=3), _stored(B, tb, pad=5)
    C = capi_gemm_ex(A_st, B_st, M, N, K, ta, tb, _cfg())
    assert_close(C, ref, K, f"pitched ({ta},{tb})")


EPILOGUES = [
    dict(alpha=0.5),
    dict(alpha=1.0, beta=1.0),
    dict(alpha=-0.75, beta=0.25, bias=True),
    dict(bias=True, act="relu"),
    dict(alpha=2.0, beta=-1.0, bias=True, act="gelu"),
    dict(act="gelu"),
]


def _epi_args(kw, M, N, seed):
    g = torch.Generator().manual_seed(seed)
    out = dict(alpha=kw.get("alpha", 1.0), beta=kw.get("beta", 0.0), act=kw.get("act", "none"))
    out["D"] = (torch.rand((M, N), generator=g) * 4 - 2).half() if out["beta"] != 0.0 else None
    out["bias"] = (torch.rand((N,), generator=g) * 2 - 1).half() if kw.get("bias") else None
    return out


@pytest.mark.parametrize("epi", EPILOGUES, ids=lambda e: "-".join(f"{k}{v}" for k, v in e.items()))
@pytest.mark.parametrize("kern", [dict(tile_n=128, stages=4), dict(tile_n=256, stages=4, mma_sm=2),
                                  dict(tile_n=512, stages=4, mma_sm=2), dict(tile_n=128, stages=4, split_k=4),
                                  dict(tile_n=64, stages=8, split_k=0)],
                         ids=lambda k: "-".join(f"{a}{b}" for a, b in k.items()))
def test_epilogue(cuda_device, epi, kern):
    M, N, K = 300, 1000, 520
    A, B = make_inputs(M, N, K, seed=len(epi) + kern["tile_n"])
    e = _epi_args(epi, M, N, seed=3)
    ref = _ref(A, B, 0, 0, alpha=e["alpha"], beta=e["beta"], D=e["D"], bias=e["bias"], activation=e["act"])
    C = capi_gemm_ex(A.cuda(), B.cuda(), M, N, K, 0, 0, _cfg(**kern), alpha=e["alpha"], beta=e["beta"],
                     D=e["D"].cuda() if e["D"] is not None else None,
                     bias=e["bias"].cuda() if e["bias"] is not None else None, act=e["act"])
    assert_close(C, ref, K, f"{epi} {kern}")


@pytest.mark.parametrize("M", [1, 16, 64])
def test_epilogue_skinny_cooperative_reduce(cuda_device, M):
    """Few rows + split-K: the cooperative reduction applies the epilogue per element."""
    N, K = 4096, 4096
    A, B = make_inputs(M, N, K, dist="skinny", seed=M)
    e = _epi_args(dict(alpha=0.5, beta=1.0, bias=True, act="gelu"), M, N, seed=M)
    ref = _ref(A, B, 0, 1, alpha=0.5, beta=1.0, D=e["D"], bias=e["bias"], activation="gelu")
    C = capi_gemm_ex(A.cuda(), B.t().contiguous().cuda(), M, N, K, 0, 1, _cfg(tile_n=128, stages=6, split_k=8),
                     alpha=0.5, beta=1.0, D=e["D"].cuda(), bias=e["bias"].cuda(), act="gelu")
    assert_close(C, ref, K, f"skinny M={M}")


def test_epilogue_in_place_and_odd_pitch(cuda_device):
    """D == C (in-place accumulate) with a C pitch TMA cannot store (st.global path)."""
    M, N, K = 130, 515, 256
    A, B = make_inputs(M, N, K, seed=9)
    Cw = (torch.rand((M, N + 3), generator=torch.Generator().manual_seed(1)) * 2 - 1).half()
    D0 = Cw[:, :N].clone()
    ref = _ref(A, B, 1, 0, alpha=1.0, beta=1.0, D=D0, bias=None, activation="none")
    Cd = Cw.cuda()
    C = Cd[:, :N]
    capi_gemm_ex(A.t().contiguous().cuda(), B.cuda(), M, N, K, 1, 0, _cfg(tile_n=256, stages=4), alpha=1.0,
                 beta=1.0, D=C, C=C)
    assert_close(C, ref, K, "in place")
    assert torch.equal(Cd[:, N:].cpu(), Cw[:, N:]), "wrote outside the C view"


def test_beta_zero_does_not_read_d_and_k_zero(cuda_device):
    M, N, K = 64, 200, 96
    A, B = make_inputs(M, N, K, seed=2)
    bias = (torch.rand((N,), generator=torch.Generator().manual_seed(4)) * 2 - 1).half()
    ref = _ref(A, B, 0, 0, alpha=1.5, bias=bias, activation="relu")
    nan_d = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    C = capi_gemm_ex(A.cuda(), B.cuda(), M, N, K, 0, 0, _cfg(), alpha=1.5, beta=0.0, D=nan_d, bias=bias.cuda(),
                     act="relu")
    assert_close(C, ref, K, "beta 0")
    # K = 0: C = act(beta * D + bias)
    D = (torch.rand((M, N), generator=torch.Generator().manual_seed(5)) * 2 - 1).half()
    A0 = torch.empty((M, 0), dtype=torch.float16, device="cuda")
    B0 = torch.empty((0, N), dtype=torch.float16, device="cuda")
    C0 = capi_gemm_ex(A0, B0, M, N, 0, 0, 0, _cfg(), alpha=3.0, beta=0.5, D=D.cuda(), bias=bias.cuda(), act="gelu")
    ref0 = oracle.gemm_ex(np.zeros((M, 0), np.float16), np.zeros((0, N), np.float16), alpha=3.0, beta=0.5,
                          D=D.numpy(), bias=bias.numpy(), activation="gelu")
    assert_close(C0, ref0, 1, "K = 0")


def test_bad_ex_arguments_rejected(cuda_device):
    from infinite_dreams import _capi
    lib = _capi.lib
    A = torch.zeros((8, 8), dtype=torch.float16, device="cuda")
    cid = _cfg()
    args = [A.data_ptr(), A.data_ptr(), A.data_ptr(), 8, 8, 8, 8, 8, 8]
    assert lib.gemm_launch_ex(*args, 2, 0, 1.0, 0.0, None, 0, None, 0, cid, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    assert lib.gemm_launch_ex(*args, 0, 0, 1.0, 0.0, None, 0, None, 7, cid, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    # beta != 0 without D
    assert lib.gemm_launch_ex(*args, 0, 0, 1.0, 1.0, None, 0, None, 0, cid, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    # stored K x M needs lda >= M
    Aw = torch.zeros((16, 4), dtype=torch.float16, device="cuda")
    st = lib.gemm_launch_ex(Aw.data_ptr(), A.data_ptr(), A.data_ptr(), 16, 8, 4, 4, 8, 8, 1, 0, 1.0, 0.0, None, 0,
                            None, 0, cid, None, 0, None)
    assert st == _capi.GEMM_ERR_INVALID_ARG and "lda >= M" in lib.gemm_last_error().decode()


def test_gemm_ex_op_reads_transposed_views_in_place(cuda_device):
    """A linear layer: y = gelu(x @ W.t() + b) with W [N, K] read K-major, no copy."""
    from infinite_dreams import infinite_dreams_ext as ext
    M, N, K = 257, 1536, 1024
    g = torch.Generator().manual_seed(11)
    x = (torch.rand((M, K), generator=g) * 2 - 1).half()
    W = (torch.rand((N, K), generator=g) * 0.1 - 0.05).half()
    b = (torch.rand((N,), generator=g) - 0.5).half()
    ref = oracle.gemm_ex(x.numpy(), W.numpy(), trans_b=True, bias=b.numpy(), activation="gelu")
    xd, Wd, bd = x.cuda(), W.cuda(), b.cuda()
    Wt = Wd.t()
    assert not Wt.is_contiguous()
    y = ext.gemm_ex(xd, Wt, bias=bd, activation="gelu")
    assert_close(y, ref, K, "linear gelu")
    # against torch's own fp32 evaluation of the same layer
    ref32 = torch.nn.functional.gelu(x.float() @ W.float().t() + b.float()).numpy()
    assert_close(y, ref32, K, "vs torch fp32")
    # in-place residual update: y = 0.5 * (xt.t() @ B) + 1.0 * y
    xt = xd.t().contiguous().t()            # an M x K view of K-major storage
    B2 = Wd[:, :N // 2].contiguous()[:K]    # [K, N/2]
    y2 = y[:, :N // 2].contiguous()
    before = y2.float().cpu().numpy()
    ref2 = oracle.gemm_ex(x.numpy(), B2.cpu().numpy(), alpha=0.5, beta=1.0, D=before.astype(np.float16))
    ext.gemm_ex(xt, B2, alpha=0.5, beta=1.0, C=y2, out=y2)
    assert_close(y2, ref2, K, "in-place residual")
    ext.check_device_errors()
