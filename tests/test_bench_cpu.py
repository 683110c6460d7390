"""bench.py helpers that need no GPU: the clock record cut to the timed
region, and the rows sampled for the oracle checks of the sharded GEMM."""
import bench


def test_clock_window_keeps_only_samples_inside_the_timed_region():
    c = bench.ClockSampler(0)
    c.max_mhz, c.source = 1965.0, "nvml"
    c.samples = [(0.5, 1965.0, 120.0, []),                    # before the region (idle)
                 (1.0, 1500.0, 900.0, ["sw_power_cap"]),
                 (1.1, 1400.0, 1000.0, []),
                 (2.5, 1965.0, 100.0, [])]                     # after the region
    w = c.window(0.95, 1.2, kernel_ms=6.8)
    assert w["samples"] == 2 and w["sm_mhz"] == 1450.0 and w["sm_mhz_min"] == 1400.0
    assert w["reasons"] == ["sw_power_cap"] and w["reason_samples"] == {"sw_power_cap": 1}
    assert w["power_w_max"] == 1000.0 and abs(w["kernel_ms_x_mhz"] - 6.8 * 1450.0) < 1e-9
    empty = c.window(3.0, 4.0)
    assert empty["samples"] == 0 and empty["sm_mhz"] is None and empty["reasons"] == ["unavailable"]


def test_sampled_rows_cover_every_block_edge():
    for world in (1, 2, 4, 8):
        blocks = bench._block_rows(16384, world, max(2, bench.PARITY_ROWS // world))
        rows = 16384 // world
        assert len(blocks) == world
        for r, b in enumerate(blocks):
            assert b[0] == r * rows and b[-1] == (r + 1) * rows - 1
            assert all(r * rows <= g < (r + 1) * rows for g in b) and b == sorted(set(b))
        assert sum(len(b) for b in blocks) >= 16


def _parity_worker(rank, world, port, q):
    """One gloo rank: its RowChecker against oracle-computed C blocks, one rank planting an error."""
    import os
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    for p in (str(root), str(root / "infinite-dreams_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import numpy as np
    import torch
    import torch.distributed as dist

    import bench
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = 256
        rows = S // world

        def block(r):
            g = torch.Generator().manual_seed(100 + r)
            return (torch.rand((rows, S), generator=g) * 2 - 1).half()

        B = (torch.rand((S, S), generator=torch.Generator().manual_seed(7)) * 2 - 1).half()
        checker = bench.RowChecker(block, B, world, rank, S, threads=1)
        full = np.concatenate([oracle.gemm_f16(block(r).numpy(), B.numpy()) for r in range(world)], 0)
        full = torch.from_numpy(full)
        mine = full[rank * rows:(rank + 1) * rows].clone()
        checks = {"local": checker.check_local(mine), "full": checker.check_full(full)}
        if rank == 1:
            bad = full.clone()
            bad[rows + 0, 5] += 1000.0      # rank 1's first row: always sampled
            checks["planted"] = checker.check_full(bad)
        else:
            checks["planted"] = checker.check_full(full)
        summary = bench._parity_summary(checks, checker, world, torch.device("cpu"))
        q.put((rank, summary))
    finally:
        dist.destroy_process_group()


def test_parity_summary_combines_every_rank_with_gloo():
    """The bench's oracle checks on two gloo ranks: correct blocks pass everywhere, and an error that only
    rank 1 sees fails the combined result on every rank."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_parity_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, summary in results.items():
        assert summary["ok"] is False, rank                      # the planted error reaches every rank
        assert summary["checks"]["local"]["ok"] and summary["checks"]["full"]["ok"], (rank, summary)
        assert not summary["checks"]["planted"]["ok"], (rank, summary)
        assert summary["rows_checked_per_gathered_c"] >= 16
