"""Per-shape dispatch: (M, N, K) -> kernel configuration, persisted as JSON.

The reference tuner searched one configuration for a fixed 5-shape set and
kept only CSV logs (infinite_dreams/tuner.py:460-558); it had no per-shape
dispatch.  Here the tuner (``tuner.py --per-shape``) writes the best knob
tuple per shape into a table, ``gemm(A, B)`` looks the shape up, and shapes
without an entry fall back to the C ABI's heuristic (``gemm_default_cfg``).

Entries store knob tuples, not menu ids, so a table survives a change of the
menu; an entry whose tuple is no longer in the menu is ignored.
"""
from __future__ import annotations

import json
import os
import threading
from pathlib import Path
from typing import Dict, Optional, Sequence, Tuple

TABLE_PATH = Path(__file__).resolve().parent / "dispatch_table.json"
ENV_TABLE = "INFINITE_DREAMS_DISPATCH_TABLE"

_lock = threading.Lock()
_cache: Dict[str, Dict[str, dict]] = {}


def shape_key(M: int, N: int, K: int) -> str:
    return f"{int(M)}x{int(N)}x{int(K)}"


def table_path(path: Optional[os.PathLike] = None) -> Path:
    if path is not None:
        return Path(path)
    return Path(os.environ.get(ENV_TABLE, str(TABLE_PATH)))


def load_table(path: Optional[os.PathLike] = None) -> Dict[str, dict]:
    p = table_path(path)
    key = str(p)
    with _lock:
        if key not in _cache:
            if p.exists():
                data = json.loads(p.read_text())
                _cache[key] = dict(data.get("shapes", {}))
            else:
                _cache[key] = {}
        return _cache[key]


def save_entry(M: int, N: int, K: int, knobs: Sequence[int], ms: float, columns: Sequence[str],
               path: Optional[os.PathLike] = None, device: str = "", extra: Optional[dict] = None) -> None:
    """Adds or replaces one shape's entry and rewrites the JSON file atomically."""
    p = table_path(path)
    with _lock:
        data = {"columns": list(columns), "shapes": {}}
        if p.exists():
            data = json.loads(p.read_text())
            data.setdefault("shapes", {})
        entry = {"knobs": [int(v) for v in knobs], "ms": float(ms),
                 "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12 if ms > 0 else None, "device": device}
        if extra:
            entry.update(extra)
        data["columns"] = list(columns)
        data["shapes"][shape_key(M, N, K)] = entry
        tmp = p.with_suffix(".json.tmp")
        tmp.write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
        os.replace(tmp, p)
        _cache.pop(str(p), None)


EPILOGUE_SUFFIX = "+epi"


def lookup(M: int, N: int, K: int, path: Optional[os.PathLike] = None, epilogue: bool = False) -> int:
    """cfg_id for a shape: the tuned entry if present and valid, else the heuristic.

    ``epilogue``: the launch has a fused epilogue that reads D or applies an
    activation.  A tuned ``MxNxK+epi`` entry is used when present.  Otherwise
    a 512-column pair tile (one TMEM accumulator, so the next tile's MMAs wait
    for the whole epilogue) is replaced by the 256-column pair tile with the
    same other knobs, whose two accumulators let the epilogue of one tile run
    under the mainloop of the next.
    """
    from . import _capi

    table = load_table(path)
    cid = -1
    if epilogue:
        entry = table.get(shape_key(M, N, K) + EPILOGUE_SUFFIX)
        if entry is not None and _capi.cfg_find(entry["knobs"]) >= 0:
            return _capi.cfg_find(entry["knobs"])
    entry = table.get(shape_key(M, N, K))
    if entry is not None:
        cid = _capi.cfg_find(entry["knobs"])
    if cid < 0:
        cid = int(_capi.lib.gemm_default_cfg(int(M), int(N), int(K)))
    if epilogue and cid >= 0:
        cols = _capi.menu_columns()
        row = _capi.menu_row(cid)
        knobs = dict(zip(cols, row))
        if knobs["tile_n"] == 512:
            knobs["tile_n"] = 256
            alt = _capi.cfg_find([knobs[c] for c in cols])
            if alt >= 0:
                return alt
    return cid


def gemm(A, B, out=None, path: Optional[os.PathLike] = None):
    """C = A @ B with the per-shape dispatched kernel configuration."""
    from . import infinite_dreams_ext as ext

    M, K = int(A.shape[0]), int(A.shape[1])
    N = int(B.shape[1])
    return ext.gemm_forward_cfg(A, B, lookup(M, N, K, path), out=out)


def entries(path: Optional[os.PathLike] = None) -> Dict[Tuple[int, int, int], dict]:
    out = {}
    for k, v in load_table(path).items():
        if k.endswith(EPILOGUE_SUFFIX):
            continue
        m, n, kk = (int(x) for x in k.split("x"))
        out[(m, n, kk)] = v
    return out
