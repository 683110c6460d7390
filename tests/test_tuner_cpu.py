"""DE tuner, projection and dispatch table on CPU (synthetic fitness)."""
import csv
import json

import numpy as np
import pytest

from infinite_dreams import dispatch, tuner
from infinite_dreams.gen_gemm_bank import COLUMNS


@pytest.fixture(scope="module")
def menu():
    return tuner.Menu()


def test_library_menu_equals_generator_menu(menu):
    assert tuner.Menu.from_library().rows == menu.rows


def test_quantize_index():
    assert tuner.quantize_index(0.49, 4) == 0
    assert tuner.quantize_index(0.5, 4) == 0      # ties to the smaller index
    assert tuner.quantize_index(1.5, 4) == 1
    assert tuner.quantize_index(1.51, 4) == 2
    assert tuner.quantize_index(-3.0, 4) == 0
    assert tuner.quantize_index(9.0, 4) == 3


def test_projection_keeps_valid_and_fixes_invalid(menu):
    good = tuner.TileConfig(128, 256, 64, 4, 1, 0, 8, 1)
    assert tuner.project_to_valid(good, menu) == good
    # 256-wide tile with 8 stages does not fit shared memory: nearest is 4 stages
    bad = tuner.TileConfig(128, 256, 64, 8, 1, 0, 8, 1)
    fixed = tuner.project_to_valid(bad, menu)
    assert menu.cfg_to_id(fixed.as_tuple()) >= 0
    assert fixed.tile_n == 256 and fixed.stages == 4
    # values off the grid snap to the grid first
    odd = tuner.TileConfig(128, 128, 64, 6, 1, 1, 3, 5)
    assert menu.cfg_to_id(tuner.project_to_valid(odd, menu).as_tuple()) >= 0


def _synthetic(cfg_id, case, opts, menu=tuner.Menu()):
    k = menu.rows[cfg_id]
    target = (128, 192, 64, 4, 1, 1, 4, 3)
    idx, tidx = tuner.to_indices(k), tuner.to_indices(target)
    return 1.0 + sum((a - b) ** 2 for a, b in zip(idx, tidx))


def _scorer(menu, tmp_path=None):
    case = tuner.BenchCase(M=1024, N=1024, K=1024, A=None, B=None)
    log = str(tmp_path / "eval.csv") if tmp_path is not None else None
    return tuner.TileScorer([case], tuner.ScoreOptions(1, 0), menu, eval_log_path=log, measure=_synthetic)


def test_de_finds_synthetic_optimum_and_is_reproducible(menu, tmp_path):
    s1 = _scorer(menu, tmp_path)
    best1, ms1, hist1 = tuner.differential_evolution_discrete(24, 25, 0.7, 0.9, s1, seed=5, verbose=False)
    s1.close()
    assert best1.as_tuple() == (128, 192, 64, 4, 1, 1, 4, 3)
    assert ms1 == 1.0
    s2 = _scorer(menu)
    best2, ms2, hist2 = tuner.differential_evolution_discrete(24, 25, 0.7, 0.9, s2, seed=5, verbose=False)
    assert best2 == best1 and [h["ms"] for h in hist2] == [h["ms"] for h in hist1]
    # history is monotone (greedy replacement)
    ms = [h["ms"] for h in hist1]
    assert all(b <= a for a, b in zip(ms, ms[1:]))
    with open(tmp_path / "eval.csv") as f:
        rows = list(csv.DictReader(f))
    assert rows and set(tuner.EVAL_FIELDS) == set(rows[0].keys())
    assert any(r["cache_hit"] == "1" for r in rows)


def test_scorer_invalid_and_cache(menu):
    s = _scorer(menu)
    bad = tuner.TileConfig(128, 96, 64, 4, 1, 0, 8, 1)
    assert s.score(bad) == tuner.TileScorer.INVALID_MS
    good = tuner.TileConfig(128, 192, 64, 4, 1, 1, 4, 3)
    assert s.score(good) == 1.0 and s.score(good) == 1.0


def test_rerank_orders_best_first(menu):
    s = _scorer(menu)
    cands = [tuner.TileConfig(128, 64, 64, 2, 1, 0, 1, 1), tuner.TileConfig(128, 192, 64, 4, 1, 1, 4, 3)]
    ranked, rows = tuner.rerank_topk(cands, s)
    assert ranked[0][0] == cands[1] and len(rows) == 2


def test_dispatch_table_round_trip(tmp_path):
    path = tmp_path / "table.json"
    from infinite_dreams import _capi
    default = dispatch.lookup(4096, 4096, 4096, path)
    assert default == _capi.lib.gemm_default_cfg(4096, 4096, 4096)
    knobs = (128, 192, 64, 3, 1, 1, 4, 1)
    dispatch.save_entry(4096, 4096, 4096, knobs, 0.1, COLUMNS, path=path, device="test")
    assert dispatch.lookup(4096, 4096, 4096, path) == _capi.cfg_find(knobs)
    data = json.loads(path.read_text())
    assert data["columns"] == list(COLUMNS)
    assert data["shapes"]["4096x4096x4096"]["knobs"] == list(knobs)
    # an entry whose tuple left the menu falls back to the heuristic
    dispatch.save_entry(8, 8, 8, (128, 96, 64, 3, 1, 1, 4, 1), 0.1, COLUMNS, path=path)
    assert dispatch.lookup(8, 8, 8, path) == _capi.lib.gemm_default_cfg(8, 8, 8)
    assert (4096, 4096, 4096) in dispatch.entries(path)


def test_committed_dispatch_table_is_valid():
    from infinite_dreams import _capi
    if not dispatch.TABLE_PATH.exists():
        pytest.skip("no committed dispatch table yet")
    for shape, entry in dispatch.entries(dispatch.TABLE_PATH).items():
        assert _capi.cfg_find(entry["knobs"]) >= 0, shape


def test_interleaved_confirmation_cancels_drift(menu):
    """Candidates measured one after the other under a drifting clock rank
    wrongly; interleaved rounds with a median rank them by their true cost."""
    true = {(128, 192, 64, 4, 1, 1, 4, 3): 1.00, (128, 256, 64, 4, 1, 0, 8, 1): 1.02}
    clock = {"t": 0}

    def drifting(cfg_id, case, opts):
        clock["t"] += 1
        # the machine slows down by 5% per measurement
        return true[menu.rows[cfg_id]] * (1.0 + 0.05 * clock["t"])

    case = tuner.BenchCase(M=8, N=8, K=8, A=None, B=None)
    cands = [tuner.TileConfig(*k) for k in true]
    s = tuner.TileScorer([case], tuner.ScoreOptions(1, 0), menu, measure=drifting)
    ranked, _ = tuner.rerank_topk(cands, s, rounds=1)
    assert ranked[0][0].as_tuple() == (128, 192, 64, 4, 1, 1, 4, 3)   # first measured wins
    clock["t"] = 0
    cands_rev = list(reversed(cands))
    s = tuner.TileScorer([case], tuner.ScoreOptions(1, 0), menu, measure=drifting)
    ranked, _ = tuner.rerank_topk(cands_rev, s, rounds=1)
    assert ranked[0][0].as_tuple() == (128, 256, 64, 4, 1, 0, 8, 1)   # order decides: biased
    clock["t"] = 0
    s = tuner.TileScorer([case], tuner.ScoreOptions(1, 0), menu, measure=drifting)
    ranked, rows = tuner.rerank_topk(cands_rev, s, rounds=4)
    assert ranked[0][0].as_tuple() == (128, 192, 64, 4, 1, 1, 4, 3)   # interleaved: the true best
    assert len(rows) == 2


def test_epilogue_lookup_prefers_double_buffered_pair_tile(tmp_path):
    from infinite_dreams import _capi
    path = tmp_path / "t.json"
    wide = (256, 512, 64, 4, 2, 1, 8, 1)
    dispatch.save_entry(8192, 8192, 8192, wide, 0.7, COLUMNS, path=path)
    assert _capi.menu_row(dispatch.lookup(8192, 8192, 8192, path)) == wide
    assert _capi.menu_row(dispatch.lookup(8192, 8192, 8192, path, epilogue=True)) == (256, 256, 64, 4, 2, 1, 8, 1)
    # a tuned epilogue entry wins
    own = (256, 256, 64, 5, 2, 0, 4, 1)
    dispatch.save_entry(8192, 8192, 8192, own, 0.75, COLUMNS, path=path)
    data = json.loads(path.read_text())
    data["shapes"]["8192x8192x8192+epi"] = data["shapes"].pop("8192x8192x8192")
    data["shapes"]["8192x8192x8192"] = {"knobs": list(wide), "ms": 0.7}
    path.write_text(json.dumps(data))
    dispatch._cache.clear()
    assert _capi.menu_row(dispatch.lookup(8192, 8192, 8192, path, epilogue=True)) == own
    assert (8192, 8192, 8192) in dispatch.entries(path) and len(dispatch.entries(path)) == 1
    # without a table entry: the heuristic, narrowed the same way
    big = dispatch.lookup(16384, 16384, 16384, tmp_path / "none.json")
    narrowed = dispatch.lookup(16384, 16384, 16384, tmp_path / "none.json", epilogue=True)
    assert _capi.menu_row(big)[1] == 512 and _capi.menu_row(narrowed)[1] == 256
