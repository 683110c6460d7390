"""Host logic of the multicast all-gather (sharded_gemm(..., exchange="multicast")) on CPU.

The GPU parts -- the symmetric-memory rendezvous that binds every rank's C
to one NVLink multicast object, the kernel's multimem stores, NCCL -- are
replaced by recording fakes.  The tests check the launch arguments (this
rank's rows at their ordinary and their multicast address), the two buffers
used in turn, that every rank refuses together when one rank has no
multicast, the C ABI's own argument checks, and the collective release.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from infinite_dreams import _capi, sharded

from test_fused_gather_cpu import FakeLib, _FakeStream, _NullContext, _zeros_cpu  # noqa: F401


class McLib(FakeLib):
    def gemm_launch_multicast(self, A, B, C, C_mc, M, N, K, lda, ldb, ldc, cfg, ws, ws_len, stream):
        self.launches.append(dict(C=C, C_mc=C_mc, M=M, N=N, K=K, ldc=ldc, cfg=cfg))
        return _capi.GEMM_OK


@pytest.fixture
def mc_world(monkeypatch):
    """A 4-rank world seen from rank 1 with fake collectives and a fake launch."""
    from infinite_dreams import infinite_dreams_ext  # noqa: F401  (reads the real menu before patching)
    lib = McLib(_capi.lib)
    calls = []
    monkeypatch.setattr(_capi, "lib", lib)
    monkeypatch.setattr(sharded.dist, "is_initialized", lambda: True)
    monkeypatch.setattr(sharded.dist, "get_world_size", lambda group=None: 4)
    monkeypatch.setattr(sharded.dist, "get_rank", lambda group=None: 1)
    monkeypatch.setattr(sharded.dist, "all_reduce", lambda t, op=None, group=None: calls.append("all_reduce"))
    monkeypatch.setattr(sharded.dist, "barrier", lambda group=None: calls.append("barrier"))
    monkeypatch.setattr(sharded, "_equal_rows", lambda rows, device, group: calls.append("equal_rows") or True)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: calls.append("synchronize"))
    sharded._mc_buffers.clear()
    yield lib, calls
    sharded._mc_buffers.clear()


def _cuda_like(monkeypatch):
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    from infinite_dreams import infinite_dreams_ext as ext
    monkeypatch.setattr(ext, "_check_inputs", lambda A, B: None)
    monkeypatch.setattr(torch.cuda, "device", lambda d: _NullContext())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda d=None: _FakeStream())
    monkeypatch.setattr(torch, "zeros", _zeros_cpu(torch.zeros))


def test_multicast_launch_arguments_and_completion(mc_world, monkeypatch):
    lib, calls = mc_world
    _cuda_like(monkeypatch)
    rows, N, K = 64, 256, 128
    made = []

    def share(r, n, d, g):
        full = torch.empty((r * 4, n), dtype=torch.float16)
        made.append((full, 0x40_0000_0000 * (len(made) + 1)))
        return full, made[-1][1], None

    monkeypatch.setattr(sharded, "_mc_share", share)
    monkeypatch.setattr(sharded, "multicast_supported", lambda d, g=None: True)
    A = torch.zeros((rows, K), dtype=torch.float16)
    B = torch.zeros((K, N), dtype=torch.float16)
    outs = [sharded.sharded_gemm(A, B, M_total=4 * rows, gather=True, exchange="multicast") for _ in range(3)]
    assert calls[-1] == "all_reduce"                      # completion after the launch
    assert calls.count("equal_rows") == 1 and len(made) == 2
    assert outs[0] is made[0][0] and outs[1] is made[1][0] and outs[2] is outs[0]   # two buffers in turn
    offset = 1 * rows * N * 2                              # rank 1's rows, in bytes
    for launch, (full, mc) in zip(lib.launches, [made[0], made[1], made[0]]):
        assert launch["C"] == full[rows:2 * rows].data_ptr()
        assert launch["C_mc"] == mc + offset
        assert launch["M"] == rows and launch["N"] == N and launch["K"] == K and launch["ldc"] == N
        knobs = _capi.menu_row(launch["cfg"])
        assert knobs[0] >= 128 and knobs[7] == 1          # no skinny tile, no split-K


def test_multicast_refused_together_and_needs_n_multiple_of_8(mc_world, monkeypatch):
    lib, calls = mc_world
    _cuda_like(monkeypatch)
    monkeypatch.setattr(sharded, "multicast_supported", lambda d, g=None: False)
    monkeypatch.setattr(sharded, "_mc_share", lambda *a: pytest.fail("no rendezvous without multicast"))
    A = torch.zeros((64, 128), dtype=torch.float16)
    with pytest.raises(sharded.MulticastUnavailable):
        sharded.sharded_gemm(A, torch.zeros((128, 256), dtype=torch.float16), gather=True, exchange="multicast")
    with pytest.raises(ValueError, match="multiple of 8"):
        sharded.sharded_gemm(A, torch.zeros((128, 252), dtype=torch.float16), gather=True, exchange="multicast")
    assert not lib.launches


class _FakeHandle:
    def __init__(self, base, mc, size, rank=1):
        self.buffer_ptrs = [0, base, 0, 0]
        self.multicast_ptr = mc
        self.buffer_size = size
        self.rank = rank


def _fake_symm(monkeypatch, mc, size_pad=0):
    import torch.distributed._symmetric_memory as symm_mem
    made = {}

    def empty(size, dtype=None, device=None):
        t = torch.empty(size, dtype=dtype)
        made["t"] = t
        return t

    def rendezvous(t, group):
        return _FakeHandle(t.data_ptr(), mc, t.numel() * 2 + size_pad)

    monkeypatch.setattr(symm_mem, "get_backend", lambda d: "CUDA")
    monkeypatch.setattr(symm_mem, "empty", empty)
    monkeypatch.setattr(symm_mem, "rendezvous", rendezvous)
    monkeypatch.setattr(sharded.dist, "group", type("G", (), {"WORLD": object()}))
    monkeypatch.setattr(torch, "tensor", _tensor_cpu(torch.tensor))
    return made


def _tensor_cpu(orig):
    def tensor(*args, **kw):
        kw.pop("device", None)
        return orig(*args, **kw)
    return tensor


def test_mc_share_returns_multicast_address_of_first_element(mc_world, monkeypatch):
    made = _fake_symm(monkeypatch, mc=0x80_0000_0000)
    full, mc, handle = sharded._mc_share(32, 64, torch.device("cpu"), None)
    assert full is made["t"] and full.shape == (128, 64) and full.dtype == torch.float16
    assert mc == 0x80_0000_0000 and handle.multicast_ptr == mc


def test_mc_share_without_multicast_mapping_raises(mc_world, monkeypatch):
    _fake_symm(monkeypatch, mc=0)
    with pytest.raises(sharded.MulticastUnavailable):
        sharded._mc_share(32, 64, torch.device("cpu"), None)


def test_release_drops_multicast_buffers_after_a_barrier(mc_world, monkeypatch):
    lib, calls = mc_world
    monkeypatch.setattr(sharded, "_mc_share", lambda r, n, d, g: (torch.empty((r * 4, n), dtype=torch.float16),
                                                                 0x1000, None))
    monkeypatch.setattr(sharded, "multicast_supported", lambda d, g=None: True)
    sharded._mc_buffer(8, 64, torch.device("cpu"), None)
    calls.clear()
    sharded.release_peer_buffers()
    assert not sharded._mc_buffers
    # every rank is past its last kernel before any drops its buffers, and all have dropped them before going on
    assert calls == ["synchronize", "barrier", "synchronize", "barrier"]


def test_capi_multicast_argument_checks():
    """The C ABI refuses these before any device work, so it runs without a GPU."""
    lib = _capi.lib
    args = dict(M=256, N=256, K=128, lda=128, ldb=256, ldc=256)

    def call(C_mc, N=256, ldc=256, C=0x10000):
        return lib.gemm_launch_multicast(0x20000, 0x30000, C, C_mc, args["M"], N, args["K"], args["lda"], N, ldc, 0,
                                         None, 0, None)

    assert call(None) == _capi.GEMM_ERR_INVALID_ARG
    assert call(0x40008) == _capi.GEMM_ERR_UNSUPPORTED          # multicast address not 16-byte aligned
    assert call(0x40000, C=0x10008) == _capi.GEMM_ERR_UNSUPPORTED
    assert call(0x40000, N=252, ldc=256) == _capi.GEMM_ERR_UNSUPPORTED
    assert call(0x40000, N=256, ldc=260) == _capi.GEMM_ERR_UNSUPPORTED


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _agree_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank 0's GPU would support multicast, rank 1's not: both must get False
        sharded._local_multicast = lambda device: rank == 0
        one = sharded.multicast_supported(torch.device("cpu"))
        sharded._local_multicast = lambda device: True
        both = sharded.multicast_supported(torch.device("cpu"))
        q.put((rank, one, both))
    finally:
        dist.destroy_process_group()


def test_two_ranks_agree_on_multicast_support():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == [(0, False, True), (1, False, True)]


def test_local_multicast_is_false_off_gpu():
    assert sharded._local_multicast(torch.device("cpu")) is False


def test_mc_share_setup_error_becomes_unavailable(mc_world, monkeypatch):
    _fake_symm(monkeypatch, mc=0x1000)
    import torch.distributed._symmetric_memory as symm_mem

    def fail(t, group):
        raise RuntimeError("multicast object could not be created")

    monkeypatch.setattr(symm_mem, "rendezvous", fail)
    with pytest.raises(sharded.MulticastUnavailable, match="could not be created"):
        sharded._mc_share(32, 64, torch.device("cpu"), None)
