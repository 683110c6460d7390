"""Timing and CSV helpers.

``time_cuda_ms`` restates the reference helper (infinite_dreams/utils.py:13-27)
with its timing bug fixed: the reference recorded start and stop on ONE event
(``start = end = torch.cuda.Event(...)``, :19), so its elapsed time was ~0.
Here start and stop are distinct events on the current stream, and an
optional L2 flush separates repetitions for shapes whose operands fit in L2,
or the repetitions are replayed from a CUDA graph (no host work between
launches).
``write_csv`` keeps the reference's field list (:30-42) and appends the
Blackwell knob columns.
"""
from __future__ import annotations

import csv
import os
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch

HISTORY_FIELDS = ["phase", "gen", "rank", "ms", "cfg_id", "tile_m", "tile_n", "tile_k", "tm", "tn"]
KNOB_FIELDS = ["stages", "mma_sm", "raster", "group", "split_k"]


def ensure_dir(path: str) -> None:
    os.makedirs(path, exist_ok=True)


_flush_buf: Dict[int, torch.Tensor] = {}


def l2_flush(device: Optional[torch.device] = None) -> None:
    """Overwrites a buffer twice the L2 size so the next kernel starts cold."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    buf = _flush_buf.get(dev)
    if buf is None:
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        buf = torch.empty(max(2 * l2, 64 << 20), dtype=torch.uint8, device=f"cuda:{dev}")
        _flush_buf[dev] = buf
    buf.fill_(1)


@torch.no_grad()
def time_cuda_ms(fn: Callable[[], Any], iters: int, warmup: int, flush_l2: bool = False,
                 graph: bool = False) -> float:
    """Mean device milliseconds of ``fn`` over ``iters`` runs after ``warmup`` runs.

    ``graph=True``: the ``iters`` calls are recorded once into a CUDA graph
    and the graph is replayed between the events, so launches follow each
    other without any host work in between (device time back to back).
    """
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        g.replay()
        end.record()
        torch.cuda.synchronize()
        del g
        return start.elapsed_time(end) / max(iters, 1)
    if not flush_l2:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / max(iters, 1)
    total = 0.0
    for _ in range(iters):
        l2_flush()
        # Keep the GPU busy (untimed) while the host enqueues fn(), so the
        # interval between the events holds only device work.
        torch.cuda._sleep(400000)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        total += start.elapsed_time(end)
    return total / max(iters, 1)


def write_csv(path: str, rows: List[Dict[str, Any]], fieldnames: Optional[Sequence[str]] = None) -> None:
    ensure_dir(os.path.dirname(path) or ".")
    fields = list(fieldnames) if fieldnames is not None else HISTORY_FIELDS + KNOB_FIELDS
    with open(path, "w", newline="", encoding="utf-8") as f:
        w = csv.DictWriter(f, fieldnames=fields, extrasaction="ignore")
        w.writeheader()
        w.writerows(rows)
