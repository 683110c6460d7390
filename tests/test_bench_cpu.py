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
