"""Per-shape throughput table: TFLOP/s and % of roofline for every workload shape.

For each shape the dispatched configuration (tuned table entry, else the
heuristic) is timed with distinct CUDA events, L2 flushed before every
repetition (``ms``: one launch per repetition, so its launch latency is
included), and back to back on warm caches (``ms_warm_b2b``, the reference
tuner's method; it includes the host work of each call), and the same back
to back replayed from a CUDA graph (``ms_graph_b2b``, device time only), on
seeded inputs (uniform[-1,1]; skinny shapes A~N(0,1), B~N(0,0.02^2)).  The roofline time of a shape is
max(2MNK / peak_flops, 2(MK+KN+MN) / peak_bw) with fp16 input/output bytes
only; % of roofline = roofline time / measured time.  Both the nominal B200
peaks (2250 TFLOP/s dense fp16, 8000 GB/s) and the measured ones
(MEASURED_PEAKS.json: bf16 GEMM burst, HBM copy) are reported.

    python -m infinite_dreams.bench_shapes [--sets single,square,skinny,irregular]
                                           [--layout nn|tn|nt|tt] [--epilogue none|bias_gelu|residual]
                                           [--torch] [--iters 20] [--out results/shapes.json]
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
from typing import Callable, Dict, List, Optional

NOMINAL_TFLOPS = 2250.0
NOMINAL_GBS = 8000.0


def measured_peaks(path: Optional[Path] = None) -> Dict[str, float]:
    p = path or Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"tflops": float(d["bf16_tflops"]), "gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"tflops": 1590.0, "gbs": 6650.0, "source": "fallback"}


def roofline_ms(M: int, N: int, K: int, tflops: float, gbs: float) -> float:
    flops = 2.0 * M * N * K
    nbytes = 2.0 * (M * K + K * N + M * N)
    return max(flops / (tflops * 1e12), nbytes / (gbs * 1e9)) * 1e3


def _shapes_of(name: str):
    """A named shape set, or an explicit shape written MxNxK."""
    from .sizes import shape_sets
    if "x" in name:
        m, n, k = (int(v) for v in name.split("x"))
        return [(m, n, k)]
    return shape_sets()[name]


EPILOGUES = ("none", "bias_gelu", "residual")


def _ops(case, layout: str, epilogue: str, cid: int, out):
    """(this build's call, torch's call) for one shape, layout and epilogue.

    layout: two letters for A and B, "n" = row-major as the reference stores
    them, "t" = stored transposed (read in place through a transposed view).
    epilogue: "none"; "bias_gelu" = gelu(A @ B + bias); "residual" =
    A @ B + C with C updated in place.  torch's call is cuBLAS (+ its own
    elementwise kernels), the same work on the same views.
    """
    import torch

    from . import infinite_dreams_ext as ext

    A = case.A.t().contiguous().t() if layout[0] == "t" else case.A
    B = case.B.t().contiguous().t() if layout[1] == "t" else case.B
    N = B.shape[1]
    if epilogue == "none":
        if layout == "nn":
            return (lambda: ext.gemm_forward_cfg(A, B, cid, out=out)), (lambda: torch.matmul(A, B, out=out))
        return (lambda: ext.gemm_ex(A, B, cfg_id=cid, out=out)), (lambda: torch.matmul(A, B, out=out))
    if epilogue == "bias_gelu":
        bias = torch.rand((N,), device=A.device, dtype=torch.float16) - 0.5
        return ((lambda: ext.gemm_ex(A, B, bias=bias, activation="gelu", cfg_id=cid, out=out)),
                (lambda: torch.nn.functional.gelu(torch.addmm(bias, A, B))))
    if epilogue == "residual":
        return ((lambda: ext.gemm_ex(A, B, beta=1.0, C=out, cfg_id=cid, out=out)),
                (lambda: out.addmm_(A, B)))
    raise ValueError(epilogue)


def run(sets: List[str], iters: int, warmup: int, cfg_override: Optional[int] = None, layout: str = "nn",
        epilogue: str = "none", with_torch: bool = False,
        check: Optional[Callable[..., Dict[str, object]]] = None,
        peaks: Optional[Dict[str, float]] = None) -> List[Dict[str, object]]:
    """One row per shape.  ``check(M, N, K, A, B, C)``, when given, is called
    once on the first result of each shape (before any timing) and its dict
    is stored under ``"parity"``; ``peaks`` ({"tflops", "gbs"}) overrides the
    measured-peak denominators."""
    import torch

    from . import dispatch, infinite_dreams_ext as ext
    from .tuner import make_bench_cases
    from .utils import time_cuda_ms

    mp = dict(peaks) if peaks is not None else measured_peaks()
    rows = []
    table = ext.gemm_cfg_table_cpu()
    seen = set()
    for name in sets:
        for (M, N, K) in _shapes_of(name):
            if (M, N, K, name) in seen:
                continue
            seen.add((M, N, K, name))
            (case,) = make_bench_cases([(M, N, K)], seed=0, dist="skinny" if name == "skinny" else "uniform")
            if cfg_override is None:
                cid = dispatch.lookup(M, N, K)
            elif cfg_override < 0:
                cid = ext.default_cfg(M, N, K)      # the C ABI's heuristic, ignoring tuned entries
            else:
                cid = cfg_override
            out = torch.zeros((M, N), dtype=torch.float16, device="cuda")
            ours, theirs = _ops(case, layout, epilogue, cid, out)
            parity = None
            if check is not None:
                out.fill_(float("nan"))
                ours()
                torch.cuda.synchronize()
                parity = check(M, N, K, case.A, case.B, out)
            ms = time_cuda_ms(ours, iters=iters, warmup=warmup, flush_l2=True)
            # back-to-back launches on warm caches, the way the reference's
            # tuner timed its kernels (infinite_dreams/utils.py:13-27)
            ms_warm = time_cuda_ms(ours, iters=iters, warmup=warmup, flush_l2=False)
            # the same launches replayed from a CUDA graph: no host work in between
            ms_graph = time_cuda_ms(ours, iters=iters, warmup=warmup, graph=True)
            ms_torch = time_cuda_ms(theirs, iters=iters, warmup=warmup, flush_l2=True) if with_torch else None
            flops = 2.0 * M * N * K
            nbytes = 2.0 * (M * K + K * N + M * N)
            rows.append({
                "set": name, "M": M, "N": N, "K": K, "layout": layout, "epilogue": epilogue, "cfg_id": cid,
                "ms_torch_cublas": ms_torch, "ms_graph_b2b": ms_graph,
                "knobs": dict(zip(ext.CFG_COLUMNS, table[cid].tolist())), "ms": ms, "ms_warm_b2b": ms_warm,
                "tflops": flops / (ms * 1e-3) / 1e12, "gbs": nbytes / (ms * 1e-3) / 1e9,
                "pct_fp16_peak_nominal": 100.0 * flops / (ms * 1e-3) / 1e12 / NOMINAL_TFLOPS,
                "pct_roofline_nominal": 100.0 * roofline_ms(M, N, K, NOMINAL_TFLOPS, NOMINAL_GBS) / ms,
                "pct_roofline_measured": 100.0 * roofline_ms(M, N, K, mp["tflops"], mp["gbs"]) / ms,
                # the same against the back-to-back time replayed from a CUDA graph: device time per
                # launch in a stream of launches, without the one launch's latency
                "pct_roofline_measured_graph": 100.0 * roofline_ms(M, N, K, mp["tflops"], mp["gbs"]) / ms_graph,
                "bound": "tensor" if flops / (NOMINAL_TFLOPS * 1e12) > nbytes / (NOMINAL_GBS * 1e9) else "hbm",
            })
            if parity is not None:
                rows[-1]["parity"] = parity
            del case, out
            torch.cuda.empty_cache()
    ext.check_device_errors()
    return rows


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sets", default="single,square,skinny,irregular",
                    help="comma-separated shape sets (single, square, skinny, irregular, default, large) or MxNxK")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cfg", type=int, default=None,
                    help="menu id for every shape; -1 = the C ABI's heuristic (default: the dispatch table)")
    ap.add_argument("--layout", default="nn", choices=["nn", "tn", "nt", "tt"],
                    help="storage of A and B: n = row-major, t = stored transposed (read in place)")
    ap.add_argument("--epilogue", default="none", choices=EPILOGUES)
    ap.add_argument("--torch", action="store_true", help="also time torch (cuBLAS) on the same views")
    ap.add_argument("--out", default="results/shapes.json")
    args = ap.parse_args(argv)
    rows = run(args.sets.split(","), args.iters, args.warmup, args.cfg, args.layout, args.epilogue, args.torch)
    os.makedirs(os.path.dirname(args.out) or ".", exist_ok=True)
    Path(args.out).write_text(json.dumps(rows, indent=1) + "\n")
    for r in rows:
        tq = f" torch {r['ms_torch_cublas']:8.4f}" if r["ms_torch_cublas"] is not None else ""
        print(f"{r['set']:9s} {r['M']:6d} {r['N']:6d} {r['K']:6d} {r['layout']} {r['epilogue']:9s} "
              f"{r['ms']:8.4f} ms (warm {r['ms_warm_b2b']:8.4f}, graph {r['ms_graph_b2b']:8.4f}){tq}  "
              f"{r['tflops']:7.1f} TF/s "
              f"{r['gbs']:7.0f} GB/s  {r['pct_roofline_nominal']:5.1f}% roof(nom) "
              f"{r['pct_roofline_measured']:5.1f}% roof(meas)  {r['bound']}  {tuple(r['knobs'].values())}")


if __name__ == "__main__":
    main()
