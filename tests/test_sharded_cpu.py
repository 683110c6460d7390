"""M-row sharding across ranks: 2 gloo ranks on CPU with a CPU GEMM stand-in."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from infinite_dreams.sharded import row_block, sharded_gemm

import oracle


def test_row_blocks_cover_rows():
    for M in (1, 7, 16, 16384, 4097):
        for world in (1, 2, 3, 4, 8):
            blocks = [row_block(M, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
            sizes = [b - a for a, b in blocks]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_compute(A, B, out):
    c = torch.from_numpy(oracle.gemm_f16(A.numpy(), B.numpy(), threads=1))
    if out is not None:
        out.copy_(c)
        return out
    return c


def _worker(rank, world, port, M, N, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        A = (torch.rand((M, K), generator=g) * 2 - 1).to(torch.float16)
        B = (torch.rand((K, N), generator=g) * 2 - 1).to(torch.float16) if rank == 0 else \
            torch.zeros((K, N), dtype=torch.float16)
        dist.broadcast(B, src=0)
        r0, r1 = row_block(M, world, rank)
        local = sharded_gemm(A[r0:r1].contiguous(), B, compute=_cpu_compute)
        full = sharded_gemm(A[r0:r1].contiguous(), B, M_total=M, gather=True, compute=_cpu_compute)
        piped = sharded_gemm(A[r0:r1].contiguous(), B, M_total=M, gather=True, compute=_cpu_compute, chunks=3)
        # the fused exchange writes into peers' GPU memory: refused for CPU tensors, and it owns its output
        errors = []
        for kw in (dict(exchange="fused"), dict(exchange="fused", compute=_cpu_compute), dict(exchange="ring")):
            try:
                sharded_gemm(A[r0:r1].contiguous(), B, M_total=M, gather=True, **kw)
                errors.append(None)
            except ValueError as e:
                errors.append(str(e))
        assert errors[0] is not None and "CUDA" in errors[0], errors
        assert errors[1] is not None and "owns its output" in errors[1], errors
        assert errors[2] is not None and "exchange must be" in errors[2], errors
        q.put((rank, local.numpy().view(np.uint16), full.numpy().view(np.uint16), (r0, r1),
               oracle.gemm_f16(A.numpy(), B.numpy()).view(np.uint16), piped.numpy().view(np.uint16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [64, 61])
def test_two_rank_sharded_gemm_matches_single(M):
    N, K, world = 48, 40, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, local, full, (r0, r1), ref, piped in results:
        assert np.array_equal(local, ref[r0:r1])
        assert np.array_equal(full, ref)
        # pipelined exchange (equal blocks) or its one-shot fallback (unequal)
        assert np.array_equal(piped, ref)
