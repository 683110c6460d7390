"""GPU tests of the host layer around the kernels: per-shape dispatch, the DE
tuner's CUDA scorer, M-row sharding on one device, and the bench contract."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_close, make_inputs, oracle_gemm

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (16, 14336, 4096), (1000, 3000, 777), (4032, 4128, 3968)])
def test_dispatch_gemm(cuda_device, M, N, K):
    """dispatch.gemm picks the tuned configuration and matches the oracle."""
    from infinite_dreams import dispatch
    A, B = make_inputs(M, N, K, seed=M + 3)
    C = dispatch.gemm(A.cuda(), B.cuda())
    assert_close(C, oracle_gemm(A, B), K, f"dispatch {M}x{N}x{K}")


def test_tuner_cuda_scorer_small_search(cuda_device, tmp_path):
    """A tiny DE search with the real CUDA scorer on one shape; the winner is
    a menu member, is persisted, and computes the right product."""
    from infinite_dreams import dispatch, infinite_dreams_ext as ext, tuner
    from infinite_dreams.gen_gemm_bank import COLUMNS
    menu = tuner.Menu.from_library()
    cases = tuner.make_bench_cases([(256, 1024, 512)], seed=1)
    scorer = tuner.TileScorer(cases, tuner.ScoreOptions(iters=3, warmup=1, flush_l2=True), menu,
                              eval_log_path=str(tmp_path / "eval.csv"))
    best, ms, hist = tuner.differential_evolution_discrete(6, 2, 0.7, 0.9, scorer, seed=3, verbose=False)
    scorer.close()
    assert menu.cfg_to_id(best.as_tuple()) >= 0 and 0 < ms < 1e3 and len(hist) == 2
    table = tmp_path / "table.json"
    dispatch.save_entry(256, 1024, 512, best.as_tuple(), ms, COLUMNS, path=table)
    cid = dispatch.lookup(256, 1024, 512, table)
    A, B = cases[0].A, cases[0].B
    assert_close(ext.gemm_forward_cfg(A, B, cid), oracle_gemm(A.cpu(), B.cpu()), 512, "tuned winner")


def test_sharded_single_rank_and_row_blocks(cuda_device):
    """sharded_gemm on one rank, and row blocks computed separately, equal the whole GEMM."""
    from infinite_dreams.sharded import row_block, sharded_gemm
    M, N, K = 1000, 768, 640
    A, B = make_inputs(M, N, K, seed=21)
    ref = oracle_gemm(A, B)
    Ad, Bd = A.cuda(), B.cuda()
    assert_close(sharded_gemm(Ad, Bd, M_total=M, gather=True), ref, K, "one rank, gathered")
    parts = []
    for r in range(3):
        r0, r1 = row_block(M, 3, r)
        parts.append(sharded_gemm(Ad[r0:r1].contiguous(), Bd))
    assert_close(torch.cat(parts, 0), ref, K, "three row blocks")


def test_bench_contract_small(cuda_device):
    """bench.py prints one JSON line with the contract's keys (small size)."""
    env = dict(os.environ, PYTHONPATH=f"{ROOT / 'infinite-dreams_b200'}:{ROOT}")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--size", "2048", "--steps", "4", "--warmup", "3",
                        "--no-cpu-baseline", "--shape-sets", "single,irregular"],
                       capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "e2e", "gpu_launches", "clocks"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 4 and d["gpu_launches"] == 4
    assert d["value"] > 50 and np.isfinite(d["roofline"]["frac"])
    assert d["e2e"]["h2d_bytes_per_step"] == 2 * (2048 * 2048 * 2) and d["e2e"]["d2h_bytes_per_step"] == 2048 * 2048 * 2
    assert d["config"]["workload"].startswith("gemm 2048x2048x2048")
    # outputs checked against the oracle: the GEMM's own C and every shape of the per-shape block
    assert d["parity"] is True, d["parity_detail"]
    assert d["shapes"]["parity"] is True and len(d["shapes"]["rows"]) == 5
    assert all(r["parity"]["ok"] for r in d["shapes"]["rows"])
    # the clock record is cut to the timed region (here too short for more than a sample or two)
    assert d["clocks"]["sampler"] in ("nvml", "nvidia-smi") and d["clocks"]["window_ms"] > 0


def test_torch_binding_matches_ctypes_path(cuda_device):
    """The compiled binding and the ctypes path launch the same kernels: identical bits."""
    import torch
    from infinite_dreams import infinite_dreams_ext as ext
    assert ext._fast is not None
    from helpers import make_inputs
    for (M, N, K) in [(300, 700, 333), (64, 4096, 4096), (1024, 1024, 1024)]:
        A, B = make_inputs(M, N, K, seed=M)
        Ad, Bd = A.cuda(), B.cuda()
        cid = ext.default_cfg(M, N, K)
        fast = ext.gemm_forward_cfg(Ad, Bd, cid)
        slow = ext._launch(Ad, Bd, cid, None)
        assert torch.equal(fast.view(torch.int16), slow.view(torch.int16)), (M, N, K)
        bias = torch.rand((N,), device="cuda").half()
        W = Bd.t().contiguous()
        y_fast = ext._fast.gemm_ex(Ad, W.t(), cid, 0.5, 0.0, None, bias, 2, None)
        ext_fast, ext._fast = ext._fast, None
        try:
            y_slow = ext.gemm_ex(Ad, W.t(), bias=bias, activation="gelu", alpha=0.5, cfg_id=cid)
        finally:
            ext._fast = ext_fast
        assert torch.equal(y_fast.view(torch.int16), y_slow.view(torch.int16)), (M, N, K)
    ext.check_device_errors()


def test_bounded_wait_times_out_and_the_context_survives(cuda_device):
    """A wait on a barrier nothing completes gives up after its limit, the host reads the error bit
    (GEMM_ERR_DEVICE_TIMEOUT), reading clears it, and GEMMs keep working on the same context."""
    import ctypes
    from infinite_dreams import _capi, infinite_dreams_ext as ext
    lib = _capi.lib
    code = ctypes.c_int(0)
    assert lib.gemm_device_error(0, ctypes.byref(code)) == _capi.GEMM_OK and code.value == 0
    waited = ctypes.c_uint64(0)
    _capi.check(lib.gemm_selftest_wait_timeout(10_000_000, ctypes.byref(waited)), "gemm_selftest_wait_timeout")
    assert 10_000_000 <= waited.value < 500_000_000, waited.value          # gave up after ~10 ms, not at once
    assert lib.gemm_device_error(0, ctypes.byref(code)) == _capi.GEMM_ERR_DEVICE_TIMEOUT
    assert code.value == 1 << 4                                            # the self-test's bit
    with pytest.raises(_capi.GemmError):                                   # the op surface reports it the same way
        lib.gemm_selftest_wait_timeout(10_000_000, ctypes.byref(waited))
        ext.check_device_errors(0)
    assert lib.gemm_device_error(0, ctypes.byref(code)) == _capi.GEMM_OK and code.value == 0
    A, B = make_inputs(256, 384, 320, seed=3)
    C = ext.gemm_forward_cfg(A.cuda(), B.cuda(), ext.default_cfg(256, 384, 320))
    assert_close(C, oracle_gemm(A, B), 320, "after a timed-out wait")
    ext.check_device_errors()
    assert lib.gemm_selftest_wait_timeout(0, ctypes.byref(waited)) == _capi.GEMM_ERR_INVALID_ARG
