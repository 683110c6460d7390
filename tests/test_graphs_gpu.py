"""The op surface recorded in CUDA graphs: replays give the bits of eager launches.

Covers a plain tile, a split-K config (workspace tickets reset by every
launch, so replays start clean), a skinny config (cluster launch) and the
fused epilogue with a transposed operand; after the static inputs change in
place, a replay recomputes from the new values.
"""
import pytest
import torch

from helpers import make_inputs

pytestmark = pytest.mark.gpu


def _cfg(knobs):
    from infinite_dreams import _capi
    cid = _capi.cfg_find(knobs)
    assert cid >= 0, knobs
    return cid


CASES = [
    ((512, 512, 512), (128, 64, 64, 6, 1, 1, 2, 1)),
    ((200, 768, 2048), (128, 128, 64, 4, 1, 0, 8, 4)),
    ((16, 4096, 4096), (16, 128, 64, 12, 1, 0, 1, 4)),
    ((1024, 1024, 1024), (256, 256, 64, 4, 2, 0, 8, 1)),
]


@pytest.mark.parametrize("shape,knobs", CASES, ids=lambda v: "x".join(map(str, v)) if len(v) == 3 else None)
def test_gemm_forward_cfg_in_a_graph(cuda_device, shape, knobs):
    from infinite_dreams import infinite_dreams_ext as ext
    M, N, K = shape
    cid = _cfg(knobs)
    A, B = make_inputs(M, N, K, seed=M + N)
    A2, B2 = make_inputs(M, N, K, seed=M + N + 1)
    Ad, Bd = A.cuda(), B.cuda()
    eager1 = ext.gemm_forward_cfg(Ad, Bd, cid).clone()
    eager2 = ext.gemm_forward_cfg(A2.cuda(), B2.cuda(), cid).clone()
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    ext.gemm_forward_cfg(Ad, Bd, cid, out=out)          # warm up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ext.gemm_forward_cfg(Ad, Bd, cid, out=out)
    for expect, (a, b) in ((eager1, (A, B)), (eager2, (A2, B2)), (eager1, (A, B))):
        Ad.copy_(a.cuda())
        Bd.copy_(b.cuda())
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), expect.view(torch.int16)), (shape, knobs)
    ext.check_device_errors()


def test_gemm_ex_epilogue_in_a_graph(cuda_device):
    """y = gelu(x @ W.t() + b) with W stored N x K, recorded once and replayed many times."""
    from infinite_dreams import infinite_dreams_ext as ext
    M, N, K = 300, 1536, 1024
    g0 = torch.Generator().manual_seed(2)
    x = ((torch.rand((M, K), generator=g0) * 2 - 1).half()).cuda()
    W = ((torch.rand((N, K), generator=g0) * 0.1 - 0.05).half()).cuda()
    b = ((torch.rand((N,), generator=g0) - 0.5).half()).cuda()
    cid = ext.default_cfg(M, N, K)
    eager = ext.gemm_ex(x, W.t(), bias=b, activation="gelu", cfg_id=cid).clone()
    y = torch.empty((M, N), dtype=torch.float16, device="cuda")
    ext.gemm_ex(x, W.t(), bias=b, activation="gelu", cfg_id=cid, out=y)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ext.gemm_ex(x, W.t(), bias=b, activation="gelu", cfg_id=cid, out=y)
    for _ in range(3):
        y.fill_(float("nan"))
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), eager.view(torch.int16))
    ext.check_device_errors()


def test_graph_timing_mode(cuda_device):
    from infinite_dreams import infinite_dreams_ext as ext
    from infinite_dreams.utils import time_cuda_ms
    A, B = make_inputs(256, 256, 256, seed=1)
    Ad, Bd = A.cuda(), B.cuda()
    out = torch.empty((256, 256), dtype=torch.float16, device="cuda")
    cid = ext.default_cfg(256, 256, 256)
    ms = time_cuda_ms(lambda: ext.gemm_forward_cfg(Ad, Bd, cid, out=out), iters=20, warmup=3, graph=True)
    assert 0.0005 < ms < 0.05, ms      # back-to-back device time of a 256^3 GEMM, in ms


@pytest.mark.parametrize("shape,knobs", [
    ((512, 512, 512), (128, 64, 64, 6, 1, 1, 2, 1)),       # main kernel, 1 CTA
    ((1024, 1024, 1024), (256, 256, 64, 4, 2, 0, 8, 1)),   # CTA pairs
    ((16, 1000, 1000), (16, 128, 64, 8, 1, 0, 1, 4)),      # skinny kernel, cluster split-K
    ((300, 777, 777), (128, 128, 64, 4, 1, 0, 8, 4)),      # unaligned pitch: pack kernel + split-K
])
def test_chained_launches_see_the_previous_result(cuda_device, shape, knobs):
    """x_{i+1} = x_i @ W on one stream with no sync in between: each launch may start its set-up under the
    previous grid (programmatic dependent launch) but must read that grid's output.  Compared bit for bit
    with the same chain synchronised after every step."""
    from infinite_dreams import infinite_dreams_ext as ext
    M, N, K = shape
    assert N == K
    cid = _cfg(knobs)
    g = torch.Generator().manual_seed(5)
    W = ((torch.rand((K, N), generator=g) * 2 - 1) / (K ** 0.5)).half().cuda()
    x0 = (torch.rand((M, K), generator=g) * 2 - 1).half().cuda()
    outs = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in range(8)]

    def chain(sync):
        x = x0
        for o in outs:
            ext.gemm_forward_cfg(x, W, cid, out=o)
            if sync:
                torch.cuda.synchronize()
            x = o
        torch.cuda.synchronize()
        return [o.clone() for o in outs]

    ref = chain(sync=True)
    for o in outs:
        o.fill_(float("nan"))
    got = chain(sync=False)
    for i, (a, b) in enumerate(zip(got, ref)):
        assert torch.isfinite(a.float()).all(), i
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), (shape, i)
    ext.check_device_errors()
