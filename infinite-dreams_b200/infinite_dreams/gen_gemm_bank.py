"""Configuration-space generator for the sm_100a FP16 GEMM kernel bank.

Replaces the reference generator src/gen_gemm_bank.py (knobs :7-30,
``smem_bytes`` :36-38, ``valid`` :41-62, ``main`` :140-271).  The reference
enumerated SIMT tiles (tile_m, tile_n, tile_k, tm, tn), capped them to 10 000
with a bucket round-robin and wrote one ``TRY_CFG`` chain per bank file.  On
Blackwell the knobs that matter are different, so the space is redefined:

===========  ==========================================================
tile_m       tile rows: 128 * mma_sm (one tcgen05 MMA of M = tile_m); or
             16 / 32 / 64 for the skinny kernel (few rows of A: the MMA
             computes C^T with 128 columns of C as its M and tile_m as its
             N; tile_n = 128, 256 or 512 columns of C per cluster (one,
             two or four MMAs per K step), split_k = K slices reduced inside a cluster
             of 1, 2, 4 or 8 CTAs through distributed shared memory)
tile_n       tile columns: one MMA N <= 256, or 512 for a CTA pair (two MMAs
             per K step, one accumulator); each CTA holds tile_n / mma_sm
             columns of B, a multiple of 64 (one 128-byte swizzle atom)
tile_k       K per pipeline stage: 64 (one 128-byte swizzle row of fp16)
stages       depth of the TMA -> shared-memory ring
mma_sm       SMs that cooperate on one MMA: 1, or 2 (a CTA pair issuing
             tcgen05 cta_group::2; no split-K, stream-K for tile_n <= 256)
raster       tile walk order: 0 = M fastest inside groups of tile-rows,
             1 = N fastest inside groups of tile-columns
group        width of those groups (L2 reuse between concurrent CTAs)
split_k      number of K slices reduced through an fp32 workspace;
             0 = stream-K (every CTA gets an equal share of all (tile, K-block)
             iterations; tiles shared by CTAs are reduced the same way)
===========  ==========================================================

Compile-time knobs (tile_n, stages, mma_sm) select one kernel instantiation; the
others are runtime parameters of that kernel.  ``cfg_id`` is the index into
the menu sorted by the knob tuple, exactly as the reference's id was the
index into its sorted capped list (src/gen_gemm_bank.py:185).

Outputs (deterministic, committed under ``csrc/generated``):

* ``gemm_cfg_menu.inc``      -- the menu rows (C array initialiser)
* ``gemm_variants.inc``      -- one ``IDB_VARIANT(BN, STAGES, CG)`` per instantiation
* ``gemm_bank_bn<BN>_sm<S>.cu`` -- explicit instantiations, one file per
                                (tile_n, mma_sm), so the bank compiles in parallel.
* ``gemm_skinny_variants.inc`` / ``gemm_bank_skinny.cu`` -- the same for the
                                skinny kernel's (tile_m, tile_n, stages) triples.
"""
from __future__ import annotations

import argparse
import itertools
from pathlib import Path
from typing import Dict, List, Sequence, Tuple

# ---------- knobs ----------
SMEM_CAP = 232448          # opt-in dynamic shared memory per CTA on sm_100 (227 KiB)
TMEM_COLS = 512            # TMEM columns per SM
BM_PER_SM = 128            # rows one tcgen05 M=128 MMA covers

TILE_MS = (16, 32, 64, 128, 256)
TILE_NS = (64, 128, 192, 256, 512)
TILE_KS = (64,)
STAGES = (2, 3, 4, 5, 6, 7, 8, 10, 12)
MMA_SMS = (1, 2)
RASTERS = (0, 1)
GROUPS = (1, 2, 4, 8, 16)
SPLIT_KS = (0, 1, 2, 3, 4, 6, 8, 12, 16)

COLUMNS = ("tile_m", "tile_n", "tile_k", "stages", "mma_sm", "raster", "group", "split_k")

# Skinny kernel (gemm_skinny_kernel.cuh): tile_m rows of A per cluster, 128
# columns of C, K split over the CTAs of a cluster.
SKINNY_TMS = (16, 32, 64)
SKINNY_NS = (128, 256, 512)
SKINNY_STAGES = (3, 4, 5, 6, 8, 10, 12)
SKINNY_SPLITS = (1, 2, 4, 8)

# Epilogue staging: 4 warps x 2 buffers x [32 rows x 64 cols] fp16.
EPI_STAGING_BYTES = 4 * 2 * 32 * 64 * 2
BARRIER_BYTES_FIXED = 5 * 8 + 16     # tmem_full[2], tmem_empty[2], done + misc words
ALIGN_SLACK = 1024

OUT_DIR = Path(__file__).resolve().parent.parent / "csrc" / "generated"
# ---------- end knobs ----------

Cfg = Tuple[int, int, int, int, int, int, int, int]


def is_skinny(tile_m: int) -> bool:
    return tile_m in SKINNY_TMS


def smem_bytes(tile_m: int, tile_n: int, tile_k: int, stages: int, mma_sm: int = 1) -> int:
    """Dynamic shared memory of one CTA; mirrors SmemPlan in gemm_sm100_kernel.cuh
    (SkinnyPlan in gemm_skinny_kernel.cuh for tile_m < 128)."""
    if is_skinny(tile_m):
        return stages * (tile_k * tile_n * 2 + tile_m * tile_k * 2) + (2 * stages + 1) * 8 + 16 + ALIGN_SLACK
    a = (tile_m // mma_sm) * tile_k * 2
    b = tile_k * (tile_n // mma_sm) * 2
    return stages * (a + b) + EPI_STAGING_BYTES + 2 * stages * 8 + BARRIER_BYTES_FIXED + ALIGN_SLACK


def tmem_cols(tile_n: int) -> int:
    # double-buffered fp32 accumulator when two fit in the 512 columns
    need = 2 * tile_n if 2 * tile_n <= TMEM_COLS else tile_n
    cols = 32
    while cols < need:
        cols *= 2
    return cols


def valid(cfg: Sequence[int]) -> bool:
    tile_m, tile_n, tile_k, stages, mma_sm, raster, group, split_k = cfg
    if is_skinny(tile_m):
        # one cluster per (tile_m x 128) block of C; raster and group do not apply
        return (tile_n in SKINNY_NS and tile_k == 64 and mma_sm == 1 and raster == 0 and group == 1
                and stages in SKINNY_STAGES and split_k in SKINNY_SPLITS
                and smem_bytes(tile_m, tile_n, tile_k, stages) <= SMEM_CAP)
    if mma_sm not in (1, 2) or tile_m != BM_PER_SM * mma_sm:
        return False
    if tile_n % (64 * mma_sm) != 0 or not (64 <= tile_n <= 256 or (tile_n == 512 and mma_sm == 2)):
        return False
    if tile_k != 64:
        return False
    if stages < 2:
        return False
    if smem_bytes(tile_m, tile_n, tile_k, stages, mma_sm) > SMEM_CAP:
        return False
    # CTA pairs: no data-parallel split-K; stream-K for the double-buffered
    # 128- and 256-column pair tiles (each CTA reduces its own 128 rows)
    if mma_sm == 2 and not (split_k == 1 or (split_k == 0 and tile_n <= 256)):
        return False
    if tmem_cols(tile_n) > TMEM_COLS:
        return False
    if raster not in (0, 1) or group < 1 or split_k < 0:
        return False
    return True


def enumerate_menu() -> List[Cfg]:
    cfgs = [c for c in itertools.product(TILE_MS, TILE_NS, TILE_KS, STAGES, MMA_SMS, RASTERS, GROUPS, SPLIT_KS)
            if valid(c)]
    cfgs.sort()
    return cfgs


def variants(menu: Sequence[Cfg]) -> List[Tuple[int, int, int]]:
    """Distinct compile-time (tile_n, stages, mma_sm) triples of the main kernel, sorted."""
    return sorted({(c[1], c[3], c[4]) for c in menu if not is_skinny(c[0])})


def skinny_variants(menu: Sequence[Cfg]) -> List[Tuple[int, int, int]]:
    """Distinct compile-time (tile_m, tile_n, stages) triples of the skinny kernel, sorted."""
    return sorted({(c[0], c[1], c[3]) for c in menu if is_skinny(c[0])})


def menu_index(menu: Sequence[Cfg]) -> Dict[Cfg, int]:
    return {c: i for i, c in enumerate(menu)}


HEADER = "// AUTO-GENERATED by infinite_dreams/gen_gemm_bank.py -- do not edit.\n"


def render(menu: Sequence[Cfg]) -> Dict[str, str]:
    out: Dict[str, str] = {}
    lines = [HEADER, f"// {len(menu)} configurations, columns: {', '.join(COLUMNS)}\n",
             f"#define IDB_MENU_COLS {len(COLUMNS)}\n",
             f"#define IDB_MENU_SIZE {len(menu)}\n",
             "static const char* const kMenuColumns[IDB_MENU_COLS] = {"
             + ", ".join(f'"{c}"' for c in COLUMNS) + "};\n",
             "static const int kMenu[IDB_MENU_SIZE][IDB_MENU_COLS] = {\n"]
    for c in menu:
        lines.append("    {" + ", ".join(str(v) for v in c) + "},\n")
    lines.append("};\n")
    out["gemm_cfg_menu.inc"] = "".join(lines)

    vs = variants(menu)
    vl = [HEADER, "// One line per compiled (tile_n, stages, mma_sm) instantiation.\n"]
    for bn, st, cg in vs:
        vl.append(f"IDB_VARIANT({bn}, {st}, {cg})\n")
    out["gemm_variants.inc"] = "".join(vl)

    sv = skinny_variants(menu)
    sl = [HEADER, "// One line per compiled (tile_m, tile_n, stages) instantiation of the skinny kernel.\n"]
    for tm, tn, st in sv:
        sl.append(f"IDB_SKINNY({tm}, {tn}, {st})\n")
    out["gemm_skinny_variants.inc"] = "".join(sl)
    bl = [HEADER, '#include "../gemm_skinny_kernel.cuh"\n\n', "namespace idb {\n"]
    for tm, tn, st in sv:
        bl.append(f"IDB_DEFINE_SKINNY({tm}, {tn}, {st})\n")
    bl.append("}  // namespace idb\n")
    out["gemm_bank_skinny.cu"] = "".join(bl)

    for bn, cg in sorted({(v[0], v[2]) for v in vs}):
        bl = [HEADER, '#include "../gemm_bank_common.cuh"\n\n', "namespace idb {\n"]
        for b2, st, c2 in vs:
            if (b2, c2) == (bn, cg):
                bl.append(f"IDB_DEFINE_VARIANT({b2}, {st}, {c2})\n")
        bl.append("}  // namespace idb\n")
        out[f"gemm_bank_bn{bn}_sm{cg}.cu"] = "".join(bl)
    return out


def write(out_dir: Path = OUT_DIR, check: bool = False) -> List[Path]:
    """Writes the generated files; with check=True only reports stale ones."""
    files = render(enumerate_menu())
    out_dir.mkdir(parents=True, exist_ok=True)
    changed: List[Path] = []
    for name, text in files.items():
        path = out_dir / name
        old = path.read_text() if path.exists() else None
        if old != text:
            changed.append(path)
            if not check:
                path.write_text(text)
    if not check:
        for stale in out_dir.glob("gemm_bank_*.cu"):
            if stale.name not in files:
                stale.unlink()
                changed.append(stale)
    return changed


def main(argv: Sequence[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--check", action="store_true", help="exit 1 if generated files are stale")
    ap.add_argument("--out", type=Path, default=OUT_DIR)
    args = ap.parse_args(argv)
    menu = enumerate_menu()
    changed = write(args.out, check=args.check)
    print(f"Generated {len(menu)} configs over {len(variants(menu)) + len(skinny_variants(menu))} kernel "
          "instantiations")
    if args.check and changed:
        print("stale:", *[str(p) for p in changed])
        raise SystemExit(1)


if __name__ == "__main__":
    main()
