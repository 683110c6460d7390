"""Generator: the Blackwell config space, its validity rules and its outputs."""
import itertools

from infinite_dreams import gen_gemm_bank as gen


def test_menu_is_sorted_unique_and_valid():
    menu = gen.enumerate_menu()
    assert menu == sorted(set(menu))
    assert len(menu) > 100
    assert all(gen.valid(c) for c in menu)


def test_valid_rules():
    ok = (128, 256, 64, 4, 1, 0, 8, 1)
    assert gen.valid(ok)
    assert not gen.valid((128, 256, 64, 5, 1, 0, 8, 1))   # shared memory above 227 KiB
    assert not gen.valid((128, 96, 64, 4, 1, 0, 8, 1))    # tile_n not a multiple of 64
    assert not gen.valid((128, 320, 64, 2, 1, 0, 8, 1))   # MMA N above 256
    assert not gen.valid((256, 128, 64, 4, 1, 0, 8, 1))   # tile_m must equal 128 * mma_sm
    assert not gen.valid((128, 128, 32, 4, 1, 0, 8, 1))   # tile_k is one 128-byte swizzle row
    assert not gen.valid((128, 128, 64, 1, 1, 0, 8, 1))   # at least double buffering
    assert not gen.valid((128, 128, 64, 4, 1, 0, 0, 1))   # group >= 1
    assert gen.valid((128, 128, 64, 4, 1, 0, 8, 0))       # split_k = 0: stream-K
    assert not gen.valid((128, 128, 64, 4, 1, 0, 8, -1))
    assert gen.valid((256, 256, 64, 4, 2, 0, 8, 0))       # stream-K for double-buffered pair tiles
    assert not gen.valid((256, 512, 64, 4, 2, 0, 8, 0))   # ... not for the single-accumulator 512 tile


def test_every_valid_combination_is_in_the_menu():
    menu = set(gen.enumerate_menu())
    for c in itertools.product(gen.TILE_MS, gen.TILE_NS, gen.TILE_KS, gen.STAGES, gen.MMA_SMS, gen.RASTERS,
                               gen.GROUPS, gen.SPLIT_KS):
        assert (c in menu) == gen.valid(c)


def test_smem_fits_and_max_stages_per_tile():
    menu = gen.enumerate_menu()
    for bn, st, sm in gen.variants(menu):
        assert gen.smem_bytes(128 * sm, bn, 64, st, sm) <= gen.SMEM_CAP
        assert gen.tmem_cols(bn) <= 512
    deepest = {(bn, sm): max(st for b, st, s in gen.variants(menu) if (b, s) == (bn, sm))
               for bn, _, sm in gen.variants(menu)}
    assert deepest == {(64, 1): 8, (128, 1): 6, (192, 1): 4, (256, 1): 4, (128, 2): 8, (256, 2): 6, (512, 2): 4}


def test_pair_rules():
    assert gen.valid((256, 256, 64, 6, 2, 0, 8, 1))
    assert not gen.valid((256, 256, 64, 6, 2, 0, 8, 2))   # no data-parallel split-K for CTA pairs
    assert gen.valid((256, 128, 64, 8, 2, 1, 4, 0))       # stream-K pairs
    assert not gen.valid((256, 192, 64, 4, 2, 0, 8, 1))   # 96 columns per CTA is not a 64-column atom
    assert not gen.valid((256, 64, 64, 4, 2, 0, 8, 1))
    assert not gen.valid((256, 256, 64, 7, 2, 0, 8, 1))   # shared memory
    assert gen.valid((256, 512, 64, 4, 2, 0, 8, 1))       # 512 columns: two MMAs, one accumulator
    assert not gen.valid((128, 512, 64, 2, 1, 0, 8, 1))   # 512 columns need a CTA pair
    assert not gen.valid((256, 512, 64, 5, 2, 0, 8, 1))


def test_generated_files_up_to_date():
    assert gen.write(check=True) == [], "csrc/generated is stale: run gen_gemm_bank.py"


def test_render_is_deterministic():
    m = gen.enumerate_menu()
    assert gen.render(m) == gen.render(list(m))


def test_skinny_rules_and_variants():
    assert gen.valid((16, 128, 64, 12, 1, 0, 1, 8))
    assert gen.valid((64, 128, 64, 8, 1, 0, 1, 1))
    assert not gen.valid((16, 128, 64, 12, 1, 0, 1, 3))   # cluster of 1, 2, 4 or 8 CTAs
    assert not gen.valid((16, 256, 64, 12, 1, 0, 1, 1))   # 128 columns of C: the TMEM lanes
    assert not gen.valid((64, 128, 64, 10, 1, 0, 1, 1))   # shared memory
    assert not gen.valid((32, 128, 64, 8, 1, 1, 1, 1))    # raster / group do not apply
    assert not gen.valid((32, 128, 64, 8, 2, 0, 1, 1))
    assert gen.valid((16, 256, 64, 6, 1, 0, 1, 2))        # two MMAs per K step
    assert not gen.valid((16, 256, 64, 8, 1, 0, 1, 2))    # shared memory
    sv = gen.skinny_variants(gen.enumerate_menu())
    deepest = {(tm, tn): max(st for a, b, st in sv if (a, b) == (tm, tn)) for tm, tn, _ in sv}
    assert deepest == {(16, 128): 12, (32, 128): 10, (64, 128): 8, (16, 256): 6, (32, 256): 6, (64, 256): 5,
                       (16, 512): 3, (32, 512): 3, (64, 512): 3}
    for tm, tn, st in sv:
        assert gen.smem_bytes(tm, tn, 64, st) <= gen.SMEM_CAP


def test_default_cfg_for_skinny_shapes():
    from infinite_dreams import _capi
    row = lambda M, N, K: _capi.menu_row(_capi.lib.gemm_default_cfg(M, N, K))
    assert row(16, 14336, 4096) == (16, 256, 64, 6, 1, 0, 1, 2)    # 56 wide blocks x 2 CTAs
    assert row(16, 4096, 4096) == (16, 128, 64, 12, 1, 0, 1, 4)    # 32 blocks x 4 CTAs
    assert row(1, 4096, 4096) == (16, 128, 64, 12, 1, 0, 1, 4)
    assert row(33, 4096, 4096) == (64, 128, 64, 8, 1, 0, 1, 4)
    assert row(64, 14336, 4096) == (64, 128, 64, 8, 1, 0, 1, 1)
    assert row(16, 2048, 8192) == (16, 128, 64, 12, 1, 0, 1, 4)    # clusters of at most 4
    assert row(7, 12288, 96) == (16, 128, 64, 12, 1, 0, 1, 1)     # 2 K blocks: no split, not wide
    assert row(65, 4096, 4096)[0] == 128                            # above 64 rows: the main kernel
