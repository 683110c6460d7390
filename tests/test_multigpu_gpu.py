"""M-row sharding across GPUs with NCCL (skipped with fewer than 2 GPUs).

Each rank computes its contiguous row block of C with the kernel bank; the
optional all-gather -- NCCL, the fused NVLink stores, or the NVSwitch
multicast stores -- assembles C, which must equal the oracle's."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    for p in (str(root), str(root / "infinite-dreams_b200"), str(root / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    import torch.distributed as dist

    from helpers import make_inputs
    from infinite_dreams.sharded import (MulticastUnavailable, broadcast_b, release_peer_buffers, row_block,
                                         sharded_gemm)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        A, B = make_inputs(M, N, K, seed=5)
        Bd = B.to(dev) if rank == 0 else torch.zeros((K, N), dtype=torch.float16, device=dev)
        broadcast_b(Bd)
        r0, r1 = row_block(M, world, rank)
        A_local = A[r0:r1].contiguous().to(dev)
        C = sharded_gemm(A_local, Bd, M_total=M, gather=True)
        torch.cuda.synchronize()
        fused = []
        if M % world == 0:
            # tiles written into every rank's C over NVLink by the GEMM itself; three calls, so that
            # one of the two alternating buffers is reused after being overwritten with NaN
            for _ in range(3):
                F = sharded_gemm(A_local, Bd, M_total=M, gather=True, exchange="fused")
                torch.cuda.synchronize()
                fused.append(F.cpu().numpy().view(np.uint16).copy())
                F.fill_(float("nan"))   # the next call must rewrite every element
        else:
            for ex in ("fused", "multicast"):
                try:
                    sharded_gemm(A_local, Bd, M_total=M, gather=True, exchange=ex)
                    fused.append(f"{ex} accepted unequal blocks")
                except ValueError:
                    pass
        # the same through one multicast store per box, when every GPU offers multicast
        mc, mc_status = [], "ran"
        if M % world == 0:
            try:
                for _ in range(3):
                    F = sharded_gemm(A_local, Bd, M_total=M, gather=True, exchange="multicast")
                    torch.cuda.synchronize()
                    mc.append(F.cpu().numpy().view(np.uint16).copy())
                    F.fill_(float("nan"))
            except MulticastUnavailable as e:
                mc_status = f"unavailable: {e}"
        q.put((rank, C.cpu().numpy().view(np.uint16), fused, mc, mc_status))
        release_peer_buffers()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [2048, 1001])
def test_sharded_gemm_nccl_allgather(cuda_device, M):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    from helpers import make_inputs, oracle_gemm
    N, K = 1536, 1024
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    A, B = make_inputs(M, N, K, seed=5)
    ref = oracle_gemm(A, B).astype(np.float32)
    tol = 1e-2 * np.sqrt(K / 1024) * np.abs(ref).max() + 1e-3
    statuses = set()
    for rank, c, fused, mc, mc_status in results:
        got = c.view(np.float16).astype(np.float32)
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= tol, rank
        for f in fused:
            assert not isinstance(f, str), f
            g = f.view(np.float16).astype(np.float32)
            assert g.shape == ref.shape and np.isfinite(g).all(), rank
            assert np.abs(g - ref).max() <= tol, ("fused", rank)
        assert len(fused) == (3 if M % world == 0 else 0)
        for f in mc:
            g = f.view(np.float16).astype(np.float32)
            assert g.shape == ref.shape and np.isfinite(g).all(), ("multicast", rank)
            assert np.abs(g - ref).max() <= tol, ("multicast", rank)
        statuses.add(mc_status)
        if M % world == 0 and mc_status == "ran":
            assert len(mc) == 3
    assert len(statuses) == 1, statuses          # every rank ran it, or every rank was refused
    if M % world == 0 and statuses != {"ran"}:
        # NCCL and fused were checked above; say that this node left the multicast exchange out
        pytest.skip(f"multicast exchange {statuses.pop()}")


def _worker_large(rank, world, port, S, q):
    """The 16384^3 workload sharded as bench.py shards it; every rank checks
    sampled rows of both gathered C's (NCCL and fused) against the oracle."""
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    for p in (str(root), str(root / "infinite-dreams_b200"), str(root / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    import torch.distributed as dist

    import oracle
    from infinite_dreams.sharded import MulticastUnavailable, broadcast_b, release_peer_buffers, sharded_gemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        rows = S // world

        def block(r):
            g = torch.Generator(device=dev)
            g.manual_seed(100 + r)
            return (torch.rand((rows, S), generator=g, device=dev) * 2 - 1).to(torch.float16)

        g = torch.Generator(device=dev)
        g.manual_seed(99)
        Bd = (torch.rand((S, S), generator=g, device=dev) * 2 - 1).to(torch.float16) if rank == 0 else \
            torch.zeros((S, S), dtype=torch.float16, device=dev)
        broadcast_b(Bd)
        A_local = block(rank)
        C = sharded_gemm(A_local, Bd, M_total=S, gather=True)
        F = sharded_gemm(A_local, Bd, M_total=S, gather=True, exchange="fused")
        try:
            Mc = sharded_gemm(A_local, Bd, M_total=S, gather=True, exchange="multicast")
        except MulticastUnavailable:
            Mc = None
        torch.cuda.synchronize()

        # first, last and two inner rows of every rank's block
        picks = [r * rows + i for r in range(world) for i in (0, rows // 3, (2 * rows) // 3, rows - 1)]
        a_rows = torch.cat([block(r)[[i - r * rows for i in picks if r * rows <= i < (r + 1) * rows]]
                            for r in range(world)], 0)
        threads = max(1, (os.cpu_count() or 1) // world)
        ref = oracle.gemm_f16(a_rows.cpu().numpy(), Bd.cpu().numpy(), threads=threads).astype(np.float32)
        tol = oracle.tolerance(ref, S)
        got_c = C[picks].float().cpu().numpy()
        got_f = F[picks].float().cpu().numpy()
        err_c = float(np.abs(got_c - ref).max()) if np.isfinite(got_c).all() else float("inf")
        err_f = float(np.abs(got_f - ref).max()) if np.isfinite(got_f).all() else float("inf")
        err_m = None
        if Mc is not None:
            got_m = Mc[picks].float().cpu().numpy()
            err_m = float(np.abs(got_m - ref).max()) if np.isfinite(got_m).all() else float("inf")
        q.put((rank, err_c, err_f, err_m, tol))
        del F, Mc
        release_peer_buffers()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def test_sharded_16384_cubed_sampled_rows(cuda_device):
    """The bench workload (16384^3, A row-sharded over every GPU, B replicated): the NCCL all-gather, the
    fused exchange and (where the GPUs offer multicast) the multicast exchange each give every rank a C
    whose sampled rows match the oracle."""
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_large, args=(r, world, port, 16384, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err_c, err_f, err_m, tol in results:
        assert err_c <= tol, ("nccl all-gather", rank, err_c, tol)
        assert err_f <= tol, ("fused exchange", rank, err_f, tol)
        assert err_m is None or err_m <= tol, ("multicast exchange", rank, err_m, tol)
    assert len({r[3] is None for r in results}) == 1   # every rank ran it or every rank was refused
