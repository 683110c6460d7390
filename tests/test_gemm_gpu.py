"""GPU parity tests: the sm_100a kernel bank through its C ABI vs the oracle.

The oracle (oracle/gemm_oracle.c) restates the reference kernel's arithmetic
(src/gemm_kernels.cuh:6-83); the acceptance bound is
|err| <= 1e-2*sqrt(K/1024)*max|C_ref| + 1e-3, written in helpers.assert_close.
C is poisoned with NaN before every launch so an unwritten tile fails.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close, capi_gemm, make_inputs, oracle_gemm

pytestmark = pytest.mark.gpu


def _ext():
    from infinite_dreams import infinite_dreams_ext
    return infinite_dreams_ext


def _cfg(tile_n=128, stages=4, raster=0, group=8, split_k=1, mma_sm=1):
    from infinite_dreams import _capi
    cid = _capi.cfg_find((128 * mma_sm, tile_n, 64, stages, mma_sm, raster, group, split_k))
    assert cid >= 0
    return cid


def _check(M, N, K, cfg_id, dist="uniform", seed=0, what=""):
    A, B = make_inputs(M, N, K, dist, seed)
    ref = oracle_gemm(A, B)
    C = capi_gemm(A.cuda(), B.cuda(), cfg_id)
    return assert_close(C, ref, K, what or f"{M}x{N}x{K} cfg {cfg_id}")


def test_single_tile_512(cuda_device):
    """The minimum slice: 512^3, uniform[-1,1] from seed 0, default config."""
    _check(512, 512, 512, _ext().default_cfg(512, 512, 512))


def test_one_tile_exact_shape(cuda_device):
    # one 128 x 128 tile, one K block: exercises descriptors without edges
    _check(128, 128, 64, _cfg(128, 4), what="128x128x64")
    _check(128, 256, 64, _cfg(256, 4), what="128x256x64")
    _check(128, 64, 128, _cfg(64, 4), what="128x64x128")


@pytest.mark.parametrize("tile_n,stages", [(64, 2), (64, 5), (64, 8), (128, 3), (128, 6), (192, 2), (192, 4),
                                           (256, 2), (256, 3), (256, 4)])
def test_every_instantiation(cuda_device, tile_n, stages):
    """Each compiled (tile_n, stages) kernel on a shape with ragged M/N/K edges."""
    _check(320, 704, 328, _cfg(tile_n, stages), seed=tile_n + stages)


@pytest.mark.parametrize("tile_n,stages", [(128, 2), (128, 5), (128, 8), (256, 2), (256, 4), (256, 6), (512, 2),
                                           (512, 3), (512, 4)])
def test_every_pair_instantiation(cuda_device, tile_n, stages):
    """CTA-pair (tcgen05 cta_group::2, 256-row tiles) kernels on ragged edges."""
    _check(320, 704, 328, _cfg(tile_n, stages, mma_sm=2), seed=100 + tile_n + stages)


@pytest.mark.parametrize("M", [100, 130, 256, 383, 520])
@pytest.mark.parametrize("tile_n", [256, 512])
def test_pair_partial_row_tiles(cuda_device, M, tile_n):
    """M=100: the odd CTA of the pair has no valid rows; M=130: two of them."""
    _check(M, 1000, 192, _cfg(tile_n, 4, mma_sm=2), seed=M)


@pytest.mark.parametrize("raster,group", [(0, 1), (0, 4), (1, 2), (1, 16)])
def test_pair_raster_orders(cuda_device, raster, group):
    _check(1100, 1536, 256, _cfg(256, 6, raster, group, mma_sm=2), seed=raster * 7 + group)
    _check(1100, 2600, 320, _cfg(512, 4, raster, group, mma_sm=2), seed=raster * 11 + group)


@pytest.mark.parametrize("raster,group", [(0, 1), (0, 16), (1, 1), (1, 4)])
def test_raster_orders(cuda_device, raster, group):
    _check(1000, 1536, 256, _cfg(128, 4, raster, group), seed=raster * 7 + group)


@pytest.mark.parametrize("split_k", [2, 3, 4, 8, 16])
def test_split_k(cuda_device, split_k):
    _check(192, 768, 2048, _cfg(128, 4, 0, 8, split_k), seed=split_k)


@pytest.mark.parametrize("M,N,K,tile_n", [(64, 4096, 4096, 128), (16, 14336, 4096, 256), (1, 4096, 4096, 64),
                                           (300, 700, 333, 128), (128, 148 * 128, 512, 128), (1000, 3000, 777, 192),
                                           (513, 1000, 64, 64), (1660, 1530, 700, 128)])
def test_stream_k(cuda_device, M, N, K, tile_n):
    """split_k = 0: every CTA takes an equal share of all (tile, K-block) iterations."""
    _check(M, N, K, _cfg(tile_n, 4, 0, 8, 0), dist="skinny", seed=M + N + K)


@pytest.mark.parametrize("M,N,K,tile_n", [(320, 704, 328, 128), (1100, 1536, 2048, 256), (100, 1000, 4096, 256),
                                           (130, 3000, 1000, 128), (2048, 2048, 2048, 256), (4096, 1024, 4096, 256),
                                           (1790, 3070, 520, 256)])
def test_stream_k_pairs(cuda_device, M, N, K, tile_n):
    """Stream-K on CTA pairs: each CTA of the pair reduces its own 128 rows (M=100: the odd CTA has none).
    1790 x 3070 (84 pair tiles: one full wave and 10 tiles) and 1660 x 1530 above (156 one-CTA tiles: 148 and
    8) take the half-empty-last-wave walk: every full wave data-parallel, the last wave's tiles in two K
    halves on twice as many workers."""
    _check(M, N, K, _cfg(tile_n, 4, 0, 8, 0, mma_sm=2), dist="skinny", seed=M + K)


def test_stream_k_pairs_large_sampled_rows(cuda_device):
    """4096^3 on stream-K pairs (256 tiles on 74 pairs: three waves data-parallel, the last 34 tiles in two K
    halves on 68 pairs), oracle on sampled rows."""
    n = 4096
    A, B = make_inputs(n, n, n, seed=7)
    C = capi_gemm(A.cuda(), B.cuda(), _cfg(256, 4, 1, 8, 0, mma_sm=2))
    rows = np.concatenate([np.random.default_rng(1).choice(n, size=40, replace=False), [0, 255, 256, n - 1]])
    assert_close(C[torch.as_tensor(rows, device=C.device)], oracle_gemm(A[rows], B), n, "4096^3 stream-K pairs")


def test_split_k_clamped_to_k_blocks(cuda_device):
    # K=100 has 2 K blocks; split 16 is clamped to 2
    _check(64, 512, 100, _cfg(128, 4, 0, 8, 16))


@pytest.mark.parametrize("M,N,K", [(1, 8, 8), (1, 1, 1), (3, 5, 7), (129, 65, 65), (17, 1000, 9)])
def test_tiny_and_odd(cuda_device, M, N, K):
    """Shapes below one tile; odd pitches take the repack + st.global paths."""
    _check(M, N, K, _ext().default_cfg(M, N, K))


def test_k_zero_gives_zeros(cuda_device):
    A = torch.empty((4, 0), dtype=torch.float16, device="cuda")
    B = torch.empty((0, 6), dtype=torch.float16, device="cuda")
    C = capi_gemm(A, B, _cfg())
    assert torch.count_nonzero(C).item() == 0


def test_pitched_operands(cuda_device):
    """Explicit pitches (views into wider buffers), aligned and unaligned."""
    M, N, K = 200, 300, 264
    A, B = make_inputs(M, N, K, seed=11)
    ref = oracle_gemm(A, B)
    for pad in (0, 8, 3):
        Aw = torch.zeros((M, K + pad), dtype=torch.float16)
        Aw[:, :K] = A
        Bw = torch.zeros((K, N + pad), dtype=torch.float16)
        Bw[:, :N] = B
        Cw = torch.full((M, N + pad), float("nan"), dtype=torch.float16, device="cuda")
        Ad, Bd = Aw.cuda(), Bw.cuda()
        capi_gemm(Ad, Bd, _cfg(), C=Cw, lda=K + pad, ldb=N + pad, ldc=N + pad, M=M, N=N, K=K)
        assert_close(Cw[:, :N], ref, K, f"pad {pad}")
        if pad:
            assert torch.isnan(Cw[:, N:].float()).all(), "wrote outside the C view"


@pytest.mark.parametrize("knobs", [(128, 4, 0, 8, 4), (64, 8, 0, 8, 0)])
def test_pitched_split_tiles(cuda_device, knobs):
    """Split-K / stream-K reduction written to a C with an odd pitch (scalar path)."""
    M, N, K = 70, 300, 520
    A, B = make_inputs(M, N, K, seed=13)
    ref = oracle_gemm(A, B)
    Cw = torch.full((M, N + 3), float("nan"), dtype=torch.float16, device="cuda")
    capi_gemm(A.cuda(), B.cuda(), _cfg(*knobs), C=Cw, ldc=N + 3, M=M, N=N, K=K)
    assert_close(Cw[:, :N], ref, K, f"split tiles, pitch {N + 3}")
    assert torch.isnan(Cw[:, N:].float()).all(), "wrote outside the C view"


def test_bad_cfg_raises(cuda_device):
    from infinite_dreams import _capi
    A = torch.zeros((8, 8), dtype=torch.float16, device="cuda")
    with pytest.raises(_capi.GemmError):
        capi_gemm(A, A, 10 ** 6)
    with pytest.raises(RuntimeError):
        _ext().gemm_forward(A, A, 128, 128, 64, 4, 4)  # the reference's (tm, tn) tail is not a menu row


@pytest.mark.parametrize("M,N,K", [(1000, 3000, 777), (4097, 1023, 2049), (333, 8191, 5120), (7, 12288, 96)])
def test_irregular_shapes(cuda_device, M, N, K):
    """Non-tile-multiple shapes with unaligned pitches (TMA OOB fill, repack, st.global)."""
    _check(M, N, K, _ext().default_cfg(M, N, K), seed=M)


@pytest.mark.parametrize("M", [1, 16, 64, 128])
@pytest.mark.parametrize("N", [4096, 14336])
def test_skinny_shapes(cuda_device, M, N):
    """Skinny decode-like shapes, A~N(0,1), B~N(0,0.02^2)."""
    _check(M, N, 4096, _ext().default_cfg(M, N, 4096), dist="skinny", seed=M + N)


@pytest.mark.parametrize("n", [256, 512, 1024, 2048])
def test_square_sweep_full(cuda_device, n):
    _check(n, n, n, _ext().default_cfg(n, n, n), seed=n)


@pytest.mark.parametrize("n", [4096, 8192, 16384])
def test_square_large_sampled_rows(cuda_device, n):
    """Large squares: full GPU GEMM, oracle on a sample of rows (exact per row)."""
    A, B = make_inputs(n, n, n, seed=n)
    C = capi_gemm(A.cuda(), B.cuda(), _ext().default_cfg(n, n, n))
    rows = np.random.default_rng(n).choice(n, size=48, replace=False)
    rows = np.concatenate([rows, [0, n - 1]])
    ref = oracle_gemm(A[rows], B)
    assert_close(C[torch.as_tensor(rows, device=C.device)], ref, n, f"{n}^3 sampled rows")
    # FP32 torch.matmul on the same rows (the other reference the workload names)
    ref32 = (A[rows].float() @ B.float()).numpy()
    assert_close(C[torch.as_tensor(rows, device=C.device)], ref32, n, f"{n}^3 vs fp32 matmul")


def test_torch_op_surface(cuda_device):
    """gemm_forward / gemm_forward_cfg / gemm_cfg_table_cpu, reference names and semantics."""
    ext = _ext()
    A, B = make_inputs(256, 384, 192, seed=5)
    ref = oracle_gemm(A, B)
    Ad, Bd = A.cuda(), B.cuda()
    table = ext.gemm_cfg_table_cpu()
    assert table.dtype == torch.int32 and table.shape == (ext.NUM_CFG, len(ext.CFG_COLUMNS))
    cid = ext.default_cfg(256, 384, 192)
    assert_close(ext.gemm_forward_cfg(Ad, Bd, cid), ref, 192, "gemm_forward_cfg")
    row = table[cid].tolist()
    assert_close(ext.gemm_forward(Ad, Bd, *row), ref, 192, "gemm_forward")
    # non-contiguous inputs are made contiguous, as the reference does
    At = Ad.t().contiguous().t()
    assert_close(ext.gemm_forward_cfg(At, Bd, cid), ref, 192, "non-contiguous A")
    with pytest.raises(RuntimeError, match="A must be float16"):
        ext.gemm_forward_cfg(Ad.float(), Bd, cid)
    with pytest.raises(RuntimeError, match="Inner dimensions must match"):
        ext.gemm_forward_cfg(Ad, Bd[:10], cid)
    with pytest.raises(RuntimeError, match="cfg_id out of range"):
        ext.gemm_forward_cfg(Ad, Bd, ext.NUM_CFG)
    ext.check_device_errors()


def _placed(X, shift, pitch):
    """X copied into a flat device buffer at element offset `shift` with row pitch `pitch`; the buffer ends
    exactly at X's last element, so no row is followed by anything of the buffer."""
    rows, cols = X.shape
    flat = torch.full((shift + (rows - 1) * pitch + cols,), float("nan"), dtype=torch.float16, device="cuda")
    view = flat.as_strided((rows, cols), (pitch, 1), shift)
    view.copy_(X.cuda())
    return view


@pytest.mark.parametrize("shift_a,pad_a,shift_b,pad_b", [(1, 1, 0, 0), (3, 5, 2, 7), (0, 0, 5, 3), (7, 1, 1, 1),
                                                         (2, 0, 6, 0), (4, 2, 0, 8)])
def test_repack_bit_identical_to_aligned(cuda_device, shift_a, pad_a, shift_b, pad_b):
    """Operands whose base or pitch TMA cannot address are repacked (aligned 16-byte loads shifted into place,
    element loads at the matrix's edges) before the GEMM: every 2-byte misalignment of the base, odd pitches,
    and matrices that end at the end of their buffer give the same bits as the aligned operands."""
    M, N, K = 333, 1000, 776
    A, B = make_inputs(M, N, K, seed=shift_a * 10 + shift_b)
    cid = _cfg(128, 4, 0, 8, 1)
    aligned = capi_gemm(A.cuda(), B.cuda(), cid)
    Ad = _placed(A, shift_a, K + pad_a)
    Bd = _placed(B, shift_b, N + pad_b)
    got = capi_gemm(Ad, Bd, cid, lda=K + pad_a, ldb=N + pad_b, M=M, N=N, K=K)
    assert torch.equal(got.view(torch.int16), aligned.view(torch.int16)), (shift_a, pad_a, shift_b, pad_b)
