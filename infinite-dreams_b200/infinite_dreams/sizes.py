"""Benchmark shape sets.

``default_sizes`` is the reference tuner's fixed 5-shape set
(infinite_dreams/sizes.py:4-11).  The other sets are the workloads the
build is measured on: square sweep, skinny decode-like shapes, irregular
non-tile-multiple shapes and the large sharded GEMM.
"""
from typing import Dict, List, Tuple

Shape = Tuple[int, int, int]


def default_sizes() -> List[Shape]:
    return [
        (4096, 4096, 4096),
        (4096, 1024, 4096),
        (1024, 4096, 4096),
        (4096, 4096, 1024),
        (4032, 4128, 3968),
    ]


def single_sizes() -> List[Shape]:
    return [(512, 512, 512)]


def square_sizes() -> List[Shape]:
    return [(n, n, n) for n in (256, 512, 1024, 2048, 4096, 8192)]


def skinny_sizes() -> List[Shape]:
    return [(m, n, 4096) for m in (1, 16, 64, 128) for n in (4096, 14336)]


def irregular_sizes() -> List[Shape]:
    return [(1000, 3000, 777), (4097, 1023, 2049), (333, 8191, 5120), (7, 12288, 96)]


def large_size() -> Shape:
    return (16384, 16384, 16384)


def sharded_sizes() -> List[Shape]:
    """Per-rank shapes of the 16384^3 GEMM row-sharded over 2, 4 and 8 ranks."""
    n = large_size()[0]
    return [(n // p, n, n) for p in (2, 4, 8)]


def shape_sets() -> Dict[str, List[Shape]]:
    return {
        "single": single_sizes(),
        "square": square_sizes(),
        "skinny": skinny_sizes(),
        "irregular": irregular_sizes(),
        "large": [large_size()],
        "sharded": sharded_sizes(),
        "default": default_sizes(),
    }
