"""Eval-log analysis (heatmap pivots, DE trajectory) on a synthetic DE run, CPU only."""
import numpy as np
import pandas as pd
import pytest

from infinite_dreams import plot_2d_heatmap, plot_de_trajectory, tuner
from infinite_dreams.gen_gemm_bank import COLUMNS


def _synthetic(cfg_id, case, opts, menu=tuner.Menu()):
    k = menu.rows[cfg_id]
    target = (128, 192, 64, 4, 1, 1, 4, 3)
    return 1.0 + sum((a - b) ** 2 for a, b in zip(tuner.to_indices(k), tuner.to_indices(target)))


@pytest.fixture(scope="module")
def eval_log(tmp_path_factory):
    path = tmp_path_factory.mktemp("log") / "eval_log.csv"
    menu = tuner.Menu()
    case = tuner.BenchCase(M=1024, N=1024, K=1024, A=None, B=None)
    s = tuner.TileScorer([case], tuner.ScoreOptions(1, 0), menu, eval_log_path=str(path), measure=_synthetic)
    tuner.differential_evolution_discrete(12, 6, 0.7, 0.9, s, seed=3, verbose=False)
    s.close()
    return path


def test_heatmap_tables_match_a_direct_reduction(eval_log, tmp_path):
    df = plot_2d_heatmap.load_eval_log(str(eval_log), "search", 1e8, collapse_by_cfg=False)
    tables = plot_2d_heatmap.facet_tables(df, "tile_n", "split_k", "stages", ["mma_sm", "raster"])
    assert tables
    for t in tables:
        sub = df
        for k, v in t["facet"].items():
            sub = sub[sub[k] == v]
        for tn in t["min_ms"].index:
            for sk in t["min_ms"].columns:
                cell = sub[(sub.tile_n == tn) & (sub.split_k == sk)]
                got = t["min_ms"].loc[tn, sk]
                if cell.empty:
                    assert np.isnan(got)
                else:
                    assert got == cell["ms"].min()
                    assert t["argmin"].loc[tn, sk] in set(cell[cell.ms == got]["stages"])
    paths = plot_2d_heatmap.write_tables(tables, str(tmp_path), "stages", png=False)
    assert len(paths) == 2 * len(tables) and all(p.endswith(".csv") for p in paths)
    back = pd.read_csv(paths[0], index_col=0)
    assert back.shape == tables[0]["min_ms"].shape


def test_heatmap_filters_sentinels_and_collapses(eval_log):
    df = plot_2d_heatmap.load_eval_log(str(eval_log), "all", 1e8, collapse_by_cfg=True)
    assert df["cfg_id"].is_unique
    assert (plot_2d_heatmap.load_eval_log(str(eval_log), "all", 2.0, False)["ms"] < 2.0).all()


def test_de_trajectory_tables(eval_log, tmp_path):
    tables = plot_de_trajectory.trajectory(pd.read_csv(eval_log))
    stats = tables["stats"]
    assert list(stats["gen"]) == sorted(stats["gen"])
    assert (stats["min"] <= stats["median"]).all() and (stats["median"] <= stats["max"]).all()
    # the per-generation minima cover every logged search evaluation
    log = pd.read_csv(eval_log)
    search = log[(log["phase"] == "search") & (log["gen"] >= 0)]
    assert stats["min"].min() == search["ms"].min()
    assert (tables["diversity"]["mean_pairwise_l2"] >= 0).all()
    assert np.isfinite(tables["points"][["pc1", "pc2"]].to_numpy()).all()
    paths = plot_de_trajectory.write(tables, str(tmp_path), png=False)
    assert len(paths) == 3


def test_pca_and_pairwise_distance_primitives():
    rng = np.random.default_rng(0)
    X = rng.normal(size=(40, 8)) * np.array([5, 3, 1, 1, 1, 1, 1, 1])
    Y = plot_de_trajectory.pca_2d(X)
    # the leading component carries the most variance, and both are uncorrelated
    assert Y[:, 0].var() >= Y[:, 1].var()
    assert abs(np.corrcoef(Y[:, 0], Y[:, 1])[0, 1]) < 1e-8
    P = rng.normal(size=(7, 3))
    brute = np.mean([np.linalg.norm(P[i] - P[j]) for i in range(7) for j in range(i + 1, 7)])
    assert plot_de_trajectory.mean_pairwise_l2(P) == pytest.approx(brute, rel=1e-10)
    assert plot_de_trajectory.mean_pairwise_l2(P[:1]) == 0.0
