"""Host logic of the fused all-gather (sharded_gemm(..., exchange="fused")) on CPU.

The GPU parts -- CUDA IPC, the kernel's NVLink stores, NCCL -- are replaced
by recording fakes, so these tests check what the host side asks of them:
the configuration it launches, the two buffers it alternates between, the
peer pointers (offset to this rank's rows) it passes, the collective it
issues after the launch, and that every mapped buffer is released.
"""
import ctypes

import pytest
import torch

from infinite_dreams import _capi, sharded


class FakeLib:
    """Stands in for the C ABI entry points the fused path calls."""

    def __init__(self, real):
        self._real = real
        self.launches = []
        self.imported = {}
        self.closed = []
        self._next = 0x7000_0000

    def gemm_ipc_export(self, ptr, handle, offset):
        handle[:8] = int(ptr).to_bytes(8, "little")
        offset._obj.value = 0
        return _capi.GEMM_OK

    def gemm_ipc_import(self, handle, offset, out):
        self._next += 0x1000_0000
        out._obj.value = self._next
        self.imported[self._next] = bytes(handle[:8])
        return _capi.GEMM_OK

    def gemm_ipc_close(self, ptr):
        self.closed.append(int(ptr))
        return _capi.GEMM_OK

    def gemm_workspace_bytes(self, *args):
        return 0

    def gemm_launch_gather(self, A, B, C, M, N, K, lda, ldb, ldc, peers, n_peers, cfg, ws, ws_len, stream):
        self.launches.append(dict(C=C, M=M, N=N, K=K, ldc=ldc, peers=[peers[i] for i in range(n_peers)], cfg=cfg))
        return _capi.GEMM_OK

    def __getattr__(self, name):
        return getattr(self._real, name)


@pytest.fixture
def fake_world(monkeypatch):
    """A 4-rank world seen from rank 1, with fake IPC / launch / collectives."""
    from infinite_dreams import infinite_dreams_ext  # noqa: F401  (reads the real menu before patching)
    lib = FakeLib(_capi.lib)
    calls = []
    monkeypatch.setattr(_capi, "lib", lib)
    monkeypatch.setattr(sharded.dist, "is_initialized", lambda: True)
    monkeypatch.setattr(sharded.dist, "get_world_size", lambda group=None: 4)
    monkeypatch.setattr(sharded.dist, "get_rank", lambda group=None: 1)

    def all_gather_object(out, obj, group=None):
        calls.append("all_gather_object")
        for r in range(len(out)):
            out[r] = (bytes([r]) * 8 + obj[0][8:], obj[1])

    def all_reduce(t, group=None):
        calls.append("all_reduce")

    monkeypatch.setattr(sharded.dist, "all_gather_object", all_gather_object)
    monkeypatch.setattr(sharded.dist, "all_reduce", all_reduce)
    monkeypatch.setattr(sharded.dist, "barrier", lambda group=None: calls.append("barrier"))
    monkeypatch.setattr(sharded, "_equal_rows", lambda rows, device, group: calls.append("equal_rows") or True)
    sharded._fused_buffers.clear()
    yield lib, calls
    sharded._fused_buffers.clear()


def test_gather_cfg_avoids_split_and_skinny_configs():
    for rows, N, K in [(2048, 16384, 16384), (16, 4096, 4096), (128, 4096, 4096), (200, 768, 2048)]:
        knobs = _capi.menu_row(sharded._gather_cfg(rows, N, K))
        assert knobs[0] >= 128 and knobs[7] == 1, (rows, knobs)


def test_fused_buffers_alternate_and_peer_pointers_are_row_offsets(fake_world, monkeypatch):
    lib, calls = fake_world
    rows, N, K = 64, 256, 128
    # CPU stand-ins for the device buffers (the launch is faked)
    monkeypatch.setattr(sharded, "_share_buffer", lambda r, n, d, g: (
        torch.empty((r * 4, n), dtype=torch.float16), [None if j == 1 else 0x1000_0000 * (j + 1) for j in range(4)]))
    fulls = []
    for _ in range(3):
        full, peers = sharded._fused_buffer(rows, N, torch.device("cpu"), None)
        fulls.append(full)
        assert peers[1] is None and all(p is not None for i, p in enumerate(peers) if i != 1)
    assert calls.count("equal_rows") == 1                      # checked once per shape
    assert fulls[0] is fulls[2] and fulls[0] is not fulls[1]   # two buffers used in turn


def test_fused_gather_launch_arguments_and_completion(fake_world, monkeypatch):
    lib, calls = fake_world
    rows, N, K = 64, 256, 128
    A = torch.zeros((rows, K), dtype=torch.float16)
    B = torch.zeros((K, N), dtype=torch.float16)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    from infinite_dreams import infinite_dreams_ext as ext
    monkeypatch.setattr(ext, "_check_inputs", lambda A, B: None)
    monkeypatch.setattr(torch.cuda, "device", lambda d: _NullContext())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda d=None: _FakeStream())

    shared = {}

    def share(r, n, d, g):
        full = torch.empty((r * 4, n), dtype=torch.float16)
        peers = [None if j == 1 else 0x1000_0000 * (j + 1) + 0x100 * len(shared) for j in range(4)]
        shared[len(shared)] = (full, peers)
        return full, peers

    monkeypatch.setattr(sharded, "_share_buffer", share)
    monkeypatch.setattr(torch, "zeros", _zeros_cpu(torch.zeros))
    out = sharded.sharded_gemm(A, B, M_total=4 * rows, gather=True, exchange="fused")
    assert calls[-1] == "all_reduce"                          # completion after the launch
    (launch,) = lib.launches
    full, peers = shared[0]
    assert out is full
    assert launch["C"] == full[rows:2 * rows].data_ptr()      # this rank's rows of its own buffer
    assert launch["M"] == rows and launch["N"] == N and launch["K"] == K and launch["ldc"] == N
    offset = 1 * rows * N * 2                                  # rank 1's rows, in bytes
    assert launch["peers"] == [p + offset for p in peers if p is not None]
    knobs = _capi.menu_row(launch["cfg"])
    assert knobs[0] >= 128 and knobs[7] == 1
    with pytest.raises(ValueError, match="expected"):
        sharded.sharded_gemm(A, B, M_total=4 * rows + 1, gather=True, exchange="fused")


def test_release_closes_every_mapping(fake_world, monkeypatch):
    lib, calls = fake_world
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    made = []

    def share(r, n, d, g):
        base = 0x1000 * (len(made) + 1)
        peers = [base + 0x10, None, base + 0x20, base + 0x30]
        made.extend(p for p in peers if p is not None)
        return torch.empty((r * 4, n), dtype=torch.float16), peers

    monkeypatch.setattr(sharded, "_share_buffer", share)
    sharded._fused_buffer(8, 64, torch.device("cpu"), None)
    sharded._fused_buffer(8, 128, torch.device("cpu"), None)
    sharded.release_peer_buffers()
    # two shapes x two buffers x three peers, each unmapped once, then a barrier
    assert len(made) == 12 and sorted(lib.closed) == sorted(made)
    assert calls[-1] == "barrier" and not sharded._fused_buffers


class _NullContext:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class _FakeStream:
    cuda_stream = 0


def _zeros_cpu(orig):
    def zeros(*args, **kw):
        kw.pop("device", None)
        return orig(*args, **kw)
    return zeros


def test_share_buffer_exchanges_handles_and_maps_every_other_rank(fake_world):
    lib, calls = fake_world
    full, peers = sharded._share_buffer(32, 64, torch.device("cpu"), None)
    assert full.shape == (128, 64) and full.dtype == torch.float16
    assert calls.count("all_gather_object") == 1
    assert peers[1] is None and len(peers) == 4
    mapped = [p for p in peers if p is not None]
    assert len(mapped) == 3 and len(set(mapped)) == 3 and set(mapped) == set(lib.imported)
    # each mapping was opened from that rank's handle (the fake tags handles with the rank)
    assert sorted(lib.imported[p][0] for p in mapped) == [0, 2, 3]


def test_more_ranks_than_peer_slots_is_refused(fake_world, monkeypatch):
    monkeypatch.setattr(sharded.dist, "get_world_size", lambda group=None: _capi.GEMM_MAX_PEERS + 2)
    with pytest.raises(ValueError, match="at most"):
        sharded._share_buffer(8, 64, torch.device("cpu"), None)
