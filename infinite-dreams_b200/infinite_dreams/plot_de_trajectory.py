"""DE search trajectory from the tuner's eval log, over the sm_100a knobs.

Follows the reference's analysis script (infinite_dreams/plot_de_trajectory.py:39-133):
filter one phase and sentinel timings, keep rows with gen >= 0, optionally
one representative (the best) row per (gen, pop_i), z-normalise the knob
vectors, and report

* the population projected on its top two principal components, coloured by
  generation (:15-21, :86-98);
* min / median / max ms per generation (:103-115);
* the mean pairwise L2 distance per generation in the normalised space, the
  population's diversity (:24-36, :120-133).

The feature vector is the eight menu knobs (the reference used its five
tuple entries, :8).  Each result is written as CSV; PNG plots are drawn as
well when matplotlib is importable.

    python -m infinite_dreams.plot_de_trajectory --csv results/eval_log.csv --outdir results/de_plots
"""
from __future__ import annotations

import argparse
import os
from typing import Dict, List, Optional

import numpy as np
import pandas as pd

from .gen_gemm_bank import COLUMNS

FEATS = list(COLUMNS)


def pca_2d(X: np.ndarray) -> np.ndarray:
    """Projection of the centred rows of X on the two leading eigenvectors of their covariance."""
    Xc = X - X.mean(axis=0, keepdims=True)
    cov = (Xc.T @ Xc) / max(1, Xc.shape[0] - 1)
    _, vecs = np.linalg.eigh(cov)          # ascending eigenvalues
    return Xc @ vecs[:, -2:][:, ::-1]      # PC1 first


def mean_pairwise_l2(X: np.ndarray) -> float:
    """Mean Euclidean distance over all unordered pairs of rows (0 for fewer than two)."""
    n = X.shape[0]
    if n <= 1:
        return 0.0
    d2 = (X * X).sum(1)[:, None] + (X * X).sum(1)[None, :] - 2.0 * X @ X.T
    d = np.sqrt(np.clip(d2, 0.0, None))
    return float(d[np.triu_indices(n, 1)].mean())


def trajectory(df: pd.DataFrame, phase: str = "search", ms_max: float = 1e8,
               pop_mode: str = "best_per_gen_popi") -> Dict[str, pd.DataFrame]:
    """The three tables: PCA points, fitness stats per generation, diversity per generation."""
    if phase != "all":
        df = df[df["phase"].astype(str).str.startswith(phase)]
    df = df[df["ms"] < ms_max]
    for col in ("gen", "pop_i"):
        if col not in df.columns:
            raise RuntimeError(f"CSV must contain a {col!r} column to trace the DE trajectory")
    df = df[df["gen"] >= 0].copy()
    if pop_mode == "best_per_gen_popi":
        df = df.sort_values("ms").groupby(["gen", "pop_i"], as_index=False).first()
    if df.empty:
        raise RuntimeError("no search rows with gen >= 0 in the eval log")
    X = df[FEATS].to_numpy(dtype=np.float64)
    mu, sd = X.mean(axis=0, keepdims=True), X.std(axis=0, keepdims=True) + 1e-6
    Xn = (X - mu) / sd
    Y = pca_2d(Xn)
    points = pd.DataFrame({"gen": df["gen"].to_numpy(), "pop_i": df["pop_i"].to_numpy(),
                           "ms": df["ms"].to_numpy(), "pc1": Y[:, 0], "pc2": Y[:, 1]})
    stats = df.groupby("gen")["ms"].agg(["min", "median", "max"]).reset_index()
    div = []
    for g, sub in df.groupby("gen", sort=True):
        Xg = (sub[FEATS].to_numpy(dtype=np.float64) - mu) / sd
        div.append({"gen": int(g), "mean_pairwise_l2": mean_pairwise_l2(Xg)})
    return {"points": points, "stats": stats, "diversity": pd.DataFrame(div)}


def _draw(tables: Dict[str, pd.DataFrame], outdir: str) -> List[str]:
    import matplotlib
    matplotlib.use("Agg")
    import matplotlib.pyplot as plt

    out = []
    p = tables["points"]
    plt.figure()
    sc = plt.scatter(p["pc1"], p["pc2"], c=p["gen"], s=18, alpha=0.7)
    plt.colorbar(sc, label="generation")
    plt.xlabel("PC1 (normalised knobs)")
    plt.ylabel("PC2")
    plt.title("DE population trajectory")
    out.append(os.path.join(outdir, "de_pca_trajectory.png"))
    plt.savefig(out[-1], dpi=180, bbox_inches="tight")
    plt.close()
    s = tables["stats"]
    plt.figure()
    for col, label in (("min", "best (min)"), ("median", "median"), ("max", "worst (max)")):
        plt.plot(s["gen"], s[col], label=label)
    plt.xlabel("generation")
    plt.ylabel("ms")
    plt.legend()
    plt.title("Population fitness vs generation")
    out.append(os.path.join(outdir, "de_fitness_stats.png"))
    plt.savefig(out[-1], dpi=180, bbox_inches="tight")
    plt.close()
    d = tables["diversity"]
    plt.figure()
    plt.plot(d["gen"], d["mean_pairwise_l2"])
    plt.xlabel("generation")
    plt.ylabel("mean pairwise distance (normalised knobs)")
    plt.title("Population diversity vs generation")
    out.append(os.path.join(outdir, "de_diversity.png"))
    plt.savefig(out[-1], dpi=180, bbox_inches="tight")
    plt.close()
    return out


def write(tables: Dict[str, pd.DataFrame], outdir: str, png: Optional[bool] = None) -> List[str]:
    os.makedirs(outdir, exist_ok=True)
    paths = []
    for name, fname in (("points", "de_pca_trajectory.csv"), ("stats", "de_fitness_stats.csv"),
                        ("diversity", "de_diversity.csv")):
        paths.append(os.path.join(outdir, fname))
        tables[name].to_csv(paths[-1], index=False)
    if png is None:
        try:
            import matplotlib  # noqa: F401
            png = True
        except ImportError:
            png = False
    if png:
        paths += _draw(tables, outdir)
    return paths


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--csv", default="results/eval_log.csv")
    ap.add_argument("--outdir", default="results/de_plots")
    ap.add_argument("--phase", default="search", choices=["search", "confirm", "all"])
    ap.add_argument("--ms_max", type=float, default=1e8)
    ap.add_argument("--pop_mode", default="best_per_gen_popi", choices=["best_per_gen_popi", "all_rows"])
    ap.add_argument("--no-png", action="store_true")
    args = ap.parse_args(argv)
    tables = trajectory(pd.read_csv(args.csv), args.phase, args.ms_max, args.pop_mode)
    paths = write(tables, args.outdir, png=False if args.no_png else None)
    print(f"Wrote {len(paths)} files to: {args.outdir}")


if __name__ == "__main__":
    main()
