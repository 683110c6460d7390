"""Heatmaps of the tuner's eval log over two knobs of the sm_100a menu.

Follows the reference's analysis script (infinite_dreams/plot_2d_heatmap.py:13-98):
read the eval log, keep one phase, drop sentinel timings (ms >= --ms_max),
optionally keep only the best row per cfg_id, then for every facet (the
reference faceted by the per-thread micro-tile (tm, tn), :43-47) reduce each
(index, columns) cell to its minimum ms over the remaining knobs and record
which value of the ``--argmin`` knob (the reference's tile_k, :55-58) reached
it.  The reference's (tm, tn) do not exist on the tcgen05 menu; the knobs that
play their role here are the CTA-pair switch and the raster order, so those are
the default facets, with tile_n x split_k as the map and stages as the argmin.

Every table is written as CSV (``<stem>_min_ms.csv``, ``<stem>_argmin_<knob>.csv``);
PNG heatmaps are drawn as well when matplotlib is importable.

    python -m infinite_dreams.plot_2d_heatmap --csv results/eval_log.csv --outdir results/heatmaps
"""
from __future__ import annotations

import argparse
import os
from typing import Dict, List, Optional, Sequence

import pandas as pd

from .gen_gemm_bank import COLUMNS


def load_eval_log(path: str, phase: str, ms_max: float, collapse_by_cfg: bool) -> pd.DataFrame:
    """The reference's filters (:24-38): phase, sentinel ms, best row per cfg_id."""
    df = pd.read_csv(path)
    if phase != "all":
        df = df[df["phase"].astype(str) == phase].copy()
    df = df[df["ms"] < ms_max].copy()
    if collapse_by_cfg:
        if "cfg_id" not in df.columns:
            raise RuntimeError("--collapse_by_cfg requires a cfg_id column")
        df = df.sort_values("ms").groupby("cfg_id", as_index=False).first()
    missing = (set(COLUMNS) | {"ms"}) - set(df.columns)
    if missing:
        raise RuntimeError(f"CSV missing columns: {sorted(missing)}")
    return df


def facet_tables(df: pd.DataFrame, index: str, columns: str, argmin: str,
                 facets: Sequence[str]) -> List[Dict[str, object]]:
    """For each facet value: pivot of min ms and pivot of the argmin knob.

    Step order as the reference (:50-61): best ms per (index, columns, argmin)
    cell first, then the argmin over ``argmin`` within each (index, columns).
    """
    out: List[Dict[str, object]] = []
    groups = [((), df)] if not facets else df.groupby(list(facets), sort=True)
    for key, sub in groups:
        if sub.empty:
            continue
        key = key if isinstance(key, tuple) else (key,)
        cell = sub.groupby([index, columns, argmin], as_index=False)["ms"].min()
        best = cell.loc[cell.groupby([index, columns])["ms"].idxmin(), [index, columns, argmin, "ms"]]
        piv_ms = best.pivot(index=index, columns=columns, values="ms").sort_index().sort_index(axis=1)
        piv_arg = best.pivot(index=index, columns=columns, values=argmin).sort_index().sort_index(axis=1)
        out.append({"facet": dict(zip(facets, (int(k) for k in key))), "min_ms": piv_ms, "argmin": piv_arg})
    return out


def _stem(facet: Dict[str, int]) -> str:
    return "heatmap" + "".join(f"_{k}{v}" for k, v in facet.items())


def _draw(piv: pd.DataFrame, label: str, title: str, path: str) -> None:
    import matplotlib
    matplotlib.use("Agg")
    import matplotlib.pyplot as plt
    import numpy as np

    plt.figure()
    im = plt.imshow(piv.to_numpy(dtype=float), aspect="auto", interpolation="nearest")
    plt.colorbar(im, label=label)
    plt.xticks(np.arange(piv.shape[1]), piv.columns.to_numpy(), rotation=90)
    plt.yticks(np.arange(piv.shape[0]), piv.index.to_numpy())
    plt.xlabel(piv.columns.name)
    plt.ylabel(piv.index.name)
    plt.title(title)
    plt.savefig(path, dpi=180, bbox_inches="tight")
    plt.close()


def write_tables(tables: List[Dict[str, object]], outdir: str, argmin: str, png: Optional[bool] = None) -> List[str]:
    """Writes each facet's two pivots as CSV (and PNG when matplotlib loads); returns the paths."""
    os.makedirs(outdir, exist_ok=True)
    if png is None:
        try:
            import matplotlib  # noqa: F401
            png = True
        except ImportError:
            png = False
    written = []
    for t in tables:
        stem = os.path.join(outdir, _stem(t["facet"]))
        tag = ", ".join(f"{k}={v}" for k, v in t["facet"].items())
        for name, piv, label in (("min_ms", t["min_ms"], f"min ms over the other knobs"),
                                 (f"argmin_{argmin}", t["argmin"], f"argmin {argmin}")):
            path = f"{stem}_{name}.csv"
            piv.to_csv(path)
            written.append(path)
            if png:
                _draw(piv, label, f"{tag}: {label}", f"{stem}_{name}.png")
                written.append(f"{stem}_{name}.png")
    return written


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--csv", default="results/eval_log.csv")
    ap.add_argument("--outdir", default="results/heatmaps")
    ap.add_argument("--ms_max", type=float, default=1e8, help="drop invalid / sentinel timings")
    ap.add_argument("--phase", default="search", choices=["search", "confirm", "all"])
    ap.add_argument("--collapse_by_cfg", action="store_true", help="keep the best row per cfg_id first")
    ap.add_argument("--index", default="tile_n", choices=COLUMNS)
    ap.add_argument("--columns", default="split_k", choices=COLUMNS)
    ap.add_argument("--argmin", default="stages", choices=COLUMNS)
    ap.add_argument("--facets", default="mma_sm,raster", help="comma-separated knobs, '' for none")
    ap.add_argument("--no-png", action="store_true")
    args = ap.parse_args(argv)
    facets = [f for f in args.facets.split(",") if f]
    for f in facets:
        if f not in COLUMNS:
            raise SystemExit(f"unknown facet knob {f!r}")
    df = load_eval_log(args.csv, args.phase, args.ms_max, args.collapse_by_cfg)
    tables = facet_tables(df, args.index, args.columns, args.argmin, facets)
    paths = write_tables(tables, args.outdir, args.argmin, png=False if args.no_png else None)
    print(f"Wrote {len(paths)} files to: {args.outdir}")


if __name__ == "__main__":
    main()
