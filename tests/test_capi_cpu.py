"""The C-ABI library loads without a GPU, exports every declared symbol, and
its host-side logic (menu, lookup, workspace sizing, argument checks) works."""
import ctypes
import re
from pathlib import Path

import pytest

from infinite_dreams import _capi, gen_gemm_bank as gen

HEADER = Path(__file__).resolve().parent.parent / "include" / "gemm_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gemm_[a-z_]+)\s*\(", text)))


def test_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(_capi.lib, n), f"{n} declared in gemm_sm100.h but not exported"
    assert sorted(_capi.symbols()) == names


def test_menu_matches_generator():
    cols, rows = _capi.menu()
    assert tuple(cols) == gen.COLUMNS
    assert rows == gen.enumerate_menu()


def test_cfg_find_round_trip():
    _, rows = _capi.menu()
    for i in (0, 1, len(rows) // 2, len(rows) - 1):
        assert _capi.cfg_find(rows[i]) == i
    assert _capi.cfg_find((128, 128, 64, 4, 4)) == -1           # the reference's 5-tuple shape
    assert _capi.cfg_find((128, 96, 64, 4, 1, 0, 8, 1)) == -1


def test_cfg_row_errors():
    buf = (ctypes.c_int * 8)()
    assert _capi.lib.gemm_cfg_row(-1, buf, 8) == _capi.GEMM_ERR_BAD_CFG
    assert _capi.lib.gemm_cfg_row(_capi.lib.gemm_num_cfgs(), buf, 8) == _capi.GEMM_ERR_BAD_CFG
    assert _capi.lib.gemm_cfg_col_name(99) is None


def _ws(a, b, M, N, K, lda, ldb, knobs):
    return _capi.lib.gemm_workspace_bytes(a, b, M, N, K, lda, ldb, _capi.cfg_find(knobs))


def test_workspace_sizing():
    cnt = _capi.lib.gemm_workspace_counter_bytes()
    assert cnt == 65536 * 4
    aligned = 1 << 20
    k1 = (128, 128, 64, 4, 1, 0, 8, 1)
    assert _ws(aligned, aligned, 4096, 4096, 4096, 4096, 4096, k1) == 0
    # split-K: tickets + (tiles * split) fp32 partial tiles
    k4 = (128, 128, 64, 4, 1, 0, 8, 4)
    tiles = 1 * 32
    assert _ws(aligned, aligned, 64, 4096, 4096, 4096, 4096, k4) == cnt + tiles * 4 * 128 * 128 * 4
    # split larger than the number of K blocks is clamped (K=128: 2 blocks)
    k16 = (128, 128, 64, 4, 1, 0, 8, 16)
    assert _ws(aligned, aligned, 64, 512, 128, 128, 512, k16) == cnt + 4 * 2 * 128 * 128 * 4
    # unaligned pitch of A (K=777): repacked into the workspace with pitch 832 (64-element rows)
    ws = _ws(aligned, aligned, 1000, 3000, 777, 777, 3000, k1)
    assert ws == cnt + ((1000 * 832 * 2 + 255) // 256) * 256
    # unaligned base address of B
    ws = _ws(aligned, aligned + 2, 64, 64, 64, 64, 64, k1)
    assert ws == cnt + 64 * 64 * 2


def _streamk_parts(num_tiles, kbt, workers):
    T = num_tiles * kbt
    owner = lambda x: ((x + 1) * workers - 1) // T
    return max(owner(t * kbt + kbt - 1) - owner(t * kbt) + 1 for t in range(num_tiles))


def test_streamk_workspace_sizing():
    """split_k = 0: stream-K over 148 workers (the B200 SM count, assumed without a GPU)."""
    cnt = _capi.lib.gemm_workspace_counter_bytes()
    aligned = 1 << 20
    ks = (128, 128, 64, 6, 1, 0, 8, 0)
    # 32 tiles x 64 K blocks over 148 workers: every tile is shared
    parts = _streamk_parts(32, 64, 148)
    assert parts >= 4
    assert _ws(aligned, aligned, 64, 4096, 4096, 4096, 4096, ks) == cnt + 32 * parts * 128 * 128 * 4
    # 148 tiles x 8 K blocks: one worker per tile, no partials, no workspace
    assert _streamk_parts(148, 8, 148) == 1
    assert _ws(aligned, aligned, 128, 148 * 128, 512, 512, 148 * 128, ks) == 0


def test_default_cfg_is_in_menu():
    for shape in [(512, 512, 512), (1, 14336, 4096), (16384, 16384, 16384), (7, 12288, 96), (1, 1, 1)]:
        cid = _capi.lib.gemm_default_cfg(*shape)
        assert 0 <= cid < _capi.lib.gemm_num_cfgs(), shape


def test_launch_argument_errors_without_gpu():
    lib = _capi.lib
    p = 1 << 20
    assert lib.gemm_launch(p, p, p, -1, 8, 8, 8, 8, 8, 0, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    assert lib.gemm_launch(p, p, p, 8, 8, 8, 4, 8, 8, 0, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    assert lib.gemm_launch(None, p, p, 8, 8, 8, 8, 8, 8, 0, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    assert lib.gemm_launch(p + 1, p, p, 8, 8, 8, 8, 8, 8, 0, None, 0, None) == _capi.GEMM_ERR_INVALID_ARG
    assert lib.gemm_launch(p, p, p, 8, 8, 8, 8, 8, 8, 10 ** 6, None, 0, None) == _capi.GEMM_ERR_BAD_CFG
    assert "out of range" in lib.gemm_last_error().decode()
    knobs = (ctypes.c_int * 8)(128, 128, 64, 4, 4, 0, 0, 0)
    assert lib.gemm_launch_knobs(p, p, p, 8, 8, 8, 8, 8, 8, knobs, 8, None, 0, None) == _capi.GEMM_ERR_BAD_CFG
    assert "not in the kernel bank menu" in lib.gemm_last_error().decode()
    # empty output is a no-op and succeeds without touching the device
    assert lib.gemm_launch(p, p, p, 0, 8, 8, 8, 8, 8, 0, None, 0, None) == _capi.GEMM_OK


def test_status_strings():
    for code, name in [(0, "GEMM_OK"), (2, "GEMM_ERR_BAD_CFG"), (6, "GEMM_ERR_DEVICE_TIMEOUT"), (42, "GEMM_ERR_UNKNOWN")]:
        assert _capi.lib.gemm_status_string(code).decode() == name


def test_reference_surface_names():
    """The torch op module exposes the reference extension's three names."""
    pytest.importorskip("torch")
    from infinite_dreams import infinite_dreams_ext as ext
    for name in ("gemm_forward", "gemm_forward_cfg", "gemm_cfg_table_cpu"):
        assert callable(getattr(ext, name))
    t = ext.gemm_cfg_table_cpu()
    assert t.dtype.is_floating_point is False and tuple(t.shape) == (ext.NUM_CFG, len(ext.CFG_COLUMNS))
    with pytest.raises(RuntimeError, match="A must be CUDA tensor"):
        import torch
        ext.gemm_forward_cfg(torch.zeros(2, 2, dtype=torch.float16), torch.zeros(2, 2, dtype=torch.float16), 0)


def test_torch_binding_loads_and_checks_on_cpu():
    """The compiled torch binding of the C ABI loads and rejects non-CUDA inputs with the reference's message."""
    import torch
    from infinite_dreams import infinite_dreams_ext as ext
    assert ext._fast is not None, "infinite_dreams/_torch_ext*.so missing: run build.py"
    for name in ("gemm_forward_cfg", "gemm_ex", "reset_workspaces"):
        assert hasattr(ext._fast, name)
    A = torch.zeros((4, 4), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="A must be CUDA tensor"):
        ext._fast.gemm_forward_cfg(A, A, 0)
    with pytest.raises(RuntimeError, match="A must be CUDA tensor"):
        ext._fast.gemm_ex(A, A, 0)


def test_streamk_splits_only_a_half_empty_last_wave():
    """256x256 pair tiles at 4096^3: 256 tiles on 74 pairs = 3 full waves + 34 tiles.  A last wave at most
    half full is the whole stream-K region (the full waves run data-parallel), shared by 68 workers: each
    of its tiles is cut into exactly two K halves, two partial slots per tile half."""
    cnt = _capi.lib.gemm_workspace_counter_bytes()
    aligned = 1 << 20
    ks = (256, 256, 64, 6, 2, 1, 16, 0)
    tiles, kbt, workers = 256, 64, 74
    region = tiles - 3 * workers              # 34 tiles
    assert _streamk_parts(region, kbt, 2 * region) == 2
    assert _ws(aligned, aligned, 4096, 4096, 4096, 4096, 4096, ks) == cnt + tiles * 2 * 2 * 128 * 256 * 4
    # a last wave more than half full (272 tiles: 3 waves + 50): the last full wave joins the region
    region = 272 - 2 * workers                # 124 tiles
    parts = _streamk_parts(region, kbt, workers)
    assert _ws(aligned, aligned, 4096, 4352, 4096, 4096, 4352, ks) == cnt + 272 * 2 * parts * 128 * 256 * 4
