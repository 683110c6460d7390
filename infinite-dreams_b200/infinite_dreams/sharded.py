"""M-row sharding of one large GEMM over the ranks of a process group.

The reference is single-GPU only.  For GEMMs too big for one GPU's time
budget (the 16384^3 workload) the rows of A are split into contiguous
blocks, one per rank (one process per GPU), B is replicated with one
broadcast, and every rank computes its own rows of C with no collective on
the data path.  The optional output exchange is an all-gather of the
contiguous C row blocks (NCCL over NVLink on GPUs, gloo on CPU in tests);
blocks are contiguous in C, so the gathered tensor needs no permutation.
With ``chunks > 1`` the exchange is pipelined with the compute: every
rank's block is cut into row chunks, each chunk's GEMM writes straight into
its rows of the full C, and that chunk's all-gather runs (asynchronously)
while the next chunk is computed.

``exchange="fused"`` folds the all-gather into the GEMM: every rank keeps a
full-size C whose memory the other ranks map once (CUDA IPC), and the
kernel's epilogue stores each finished tile both locally and, over NVLink,
into every peer's copy (``gemm_launch_gather``), so the transfer overlaps
the remaining tiles' mainloop.  A one-element NCCL all-reduce issued after
the launch on the same stream marks the point where every rank's grid, and
with it every write into this rank's C, has completed.  No kernel reads
another GPU's memory; peers are only written to.

``exchange="multicast"`` is the same exchange through NVSwitch multicast
(NVLS): every rank's full C is bound to one multicast object (torch's
symmetric memory sets it up), and the kernel stores each finished box once,
at its multicast address, with ``multimem.st``; the switch writes it into
every rank's copy (``gemm_launch_multicast``).  Each GPU then sends its
block of C once instead of once per peer, so at 8 ranks the GEMM's own SMs
issue 1/7 of the outgoing stores.  It needs GPUs that support multicast
(``multicast_supported``).
"""
from __future__ import annotations

import ctypes
import threading
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist


def row_block(M: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank's rows: blocks differ by at most one row, larger first."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    base, rem = divmod(M, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def broadcast_b(B: torch.Tensor, src: int = 0, group=None) -> torch.Tensor:
    """Replicates B from `src` to every rank (in place)."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.broadcast(B, src=src, group=group)
    return B


def _default_compute(A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    from . import dispatch
    return dispatch.gemm(A, B, out=out)


def sharded_gemm(A_local: torch.Tensor, B: torch.Tensor, M_total: Optional[int] = None, gather: bool = False,
                 group=None, out: Optional[torch.Tensor] = None,
                 compute: Optional[Callable[[torch.Tensor, torch.Tensor, Optional[torch.Tensor]], torch.Tensor]] = None,
                 chunks: int = 1, exchange: str = "nccl") -> torch.Tensor:
    """This rank's rows of C = A @ B (or all of C when gather=True).

    A_local holds this rank's row block (``row_block``); B is the full
    replicated K x N operand.  ``compute`` defaults to the dispatched
    kernel-bank GEMM.  ``chunks`` > 1 overlaps the all-gather with the
    compute (equal row blocks only; other cases fall back to one exchange).
    ``exchange="fused"`` (gather=True, CUDA, equal row blocks) writes every
    tile to all ranks from inside the GEMM; the returned full C is a buffer
    owned by this module: it stays intact until the second fused call of
    that shape after this one, provided whatever reads it is issued on the
    calling stream before the next fused call.  ``exchange="multicast"``
    does the same through one NVSwitch multicast store per box (N a
    multiple of 8); it raises ``MulticastUnavailable`` on every rank when
    some rank's GPU has no multicast.
    """
    if exchange not in ("nccl", "fused", "multicast"):
        raise ValueError("exchange must be 'nccl', 'fused' or 'multicast'")
    if exchange != "nccl" and gather and dist.is_initialized() and dist.get_world_size(group) > 1:
        if out is not None or compute is not None:
            raise ValueError(f"exchange='{exchange}' owns its output buffer and runs the kernel bank itself")
        return _fused_gather(A_local, B, M_total, group, multicast=exchange == "multicast")
    compute = compute or _default_compute
    if gather and chunks > 1 and dist.is_initialized() and dist.get_world_size(group) > 1:
        full = _pipelined_gather(A_local, B, M_total, group, out, compute, chunks)
        if full is not None:
            return full
    C_local = compute(A_local, B, None if gather else out)
    if not gather:
        return C_local
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        if out is not None:
            out.copy_(C_local)
            return out
        return C_local
    rank = dist.get_rank(group)
    M = int(M_total) if M_total is not None else None
    sizes = torch.tensor([C_local.shape[0]], device=C_local.device, dtype=torch.int64)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes, group=group)
    rows = [int(s.item()) for s in all_sizes]
    if M is not None and sum(rows) != M:
        raise ValueError(f"row blocks sum to {sum(rows)}, expected {M}")
    mx = max(rows)
    N = C_local.shape[1]
    if all(r == mx for r in rows):
        full = out if out is not None else torch.empty((mx * world, N), dtype=C_local.dtype, device=C_local.device)
        dist.all_gather_into_tensor(full, C_local.contiguous(), group=group)
        return full
    # uneven blocks: gather padded blocks, then compact (rank order = row order)
    padded = torch.zeros((mx, N), dtype=C_local.dtype, device=C_local.device)
    padded[: rows[rank]] = C_local
    buf = torch.empty((mx * world, N), dtype=C_local.dtype, device=C_local.device)
    dist.all_gather_into_tensor(buf, padded, group=group)
    parts = [buf[r * mx: r * mx + rows[r]] for r in range(world)]
    full = torch.cat(parts, 0)
    if out is not None:
        out.copy_(full)
        return out
    return full


def _pipelined_gather(A_local: torch.Tensor, B: torch.Tensor, M_total: Optional[int], group,
                      out: Optional[torch.Tensor], compute, chunks: int) -> Optional[torch.Tensor]:
    """Chunked compute + all-gather; None when the row blocks are unequal."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows = int(A_local.shape[0])
    sizes = torch.tensor([rows], device=A_local.device, dtype=torch.int64)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes, group=group)
    if any(int(s.item()) != rows for s in all_sizes):
        return None
    M = rows * world
    if M_total is not None and int(M_total) != M:
        raise ValueError(f"row blocks sum to {M}, expected {M_total}")
    N = int(B.shape[1])
    full = out if out is not None else torch.empty((M, N), dtype=torch.float16, device=A_local.device)
    bounds = [rows * c // chunks for c in range(chunks + 1)]
    works = []
    for c in range(chunks):
        c0, c1 = bounds[c], bounds[c + 1]
        if c1 == c0:
            continue
        mine = full[rank * rows + c0: rank * rows + c1]
        compute(A_local[c0:c1].contiguous(), B, mine)
        outs = [full[r * rows + c0: r * rows + c1] for r in range(world)]
        works.append(dist.all_gather(outs, mine, group=group, async_op=True))
    for w in works:
        w.wait()
    return full


# ---------------------------------------------------------------- fused all-gather

_ipc_lock = threading.Lock()
# (rows, N, device, group key) -> two (full C buffer, [peer base pointer or None per rank]) pairs used
# alternately, and the index of the next one
_fused_buffers: Dict[Tuple[int, int, int, int], list] = {}
# the same for the multicast exchange: two (full C buffer, multicast address of its first element,
# symmetric-memory handle) triples used alternately, and the index of the next one
_mc_buffers: Dict[Tuple[int, int, int, int], list] = {}


class MulticastUnavailable(RuntimeError):
    """Raised on every rank when some rank's GPU offers no NVLink multicast."""


def _local_multicast(device: torch.device) -> bool:
    """Whether this rank's GPU supports NVLink multicast."""
    if device.type != "cuda":
        return False
    try:
        from torch._C._distributed_c10d import _SymmetricMemory
        from torch.distributed._symmetric_memory import DeviceType

        return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index))
    except (ImportError, AttributeError, RuntimeError):
        return False


def multicast_supported(device: torch.device, group=None) -> bool:
    """Whether every rank's GPU supports NVLink multicast (collective: every rank calls it)."""
    flag = torch.tensor([int(_local_multicast(device))], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(int(flag.item()))


def _group_key(group) -> int:
    return 0 if group is None else id(group)


def _equal_rows(rows: int, device: torch.device, group) -> bool:
    world = dist.get_world_size(group)
    sizes = torch.tensor([rows], device=device, dtype=torch.int64)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes, group=group)
    return all(int(s.item()) == rows for s in all_sizes)


def _fused_buffer(rows: int, N: int, device: torch.device, group) -> Tuple[torch.Tensor, List[Optional[int]]]:
    """This rank's full C for the next fused call and the other ranks' copies of it, mapped here.

    Two buffers per shape are used in turn.  Peers write a call's tiles into
    this rank's buffer while this rank may still be reading the previous
    call's result; the buffer they write was last read before the previous
    call's closing all-reduce, which every rank's stream has passed before
    any peer's kernel of this call starts.  So a result stays intact until
    the call after next, provided work that reads it is issued on the calling
    stream before the next fused call.

    The buffers are set up on the first call for a shape, which also checks
    (collectively) that every rank has the same number of rows; later calls
    of that shape take no collective step here, so every rank must keep
    passing equal row blocks."""
    key = (rows, N, device.index, _group_key(group))
    with _ipc_lock:
        entry = _fused_buffers.get(key)
    if entry is None:
        if not _equal_rows(rows, device, group):
            raise ValueError("exchange='fused' needs equal row blocks on every rank")
        entry = [_share_buffer(rows, N, device, group), _share_buffer(rows, N, device, group), 0]
        with _ipc_lock:
            _fused_buffers[key] = entry
    pair = entry[entry[2]]
    entry[2] ^= 1
    return pair


def _share_buffer(rows: int, N: int, device: torch.device, group) -> Tuple[torch.Tensor, List[Optional[int]]]:
    """A new full-size C on this rank, and every other rank's one mapped into this process."""
    from . import _capi

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if world - 1 > _capi.GEMM_MAX_PEERS:
        raise ValueError(f"the fused all-gather supports at most {_capi.GEMM_MAX_PEERS + 1} ranks")
    full = torch.empty((rows * world, N), dtype=torch.float16, device=device)
    handle = (ctypes.c_char * _capi.GEMM_IPC_HANDLE_BYTES)()
    offset = ctypes.c_int64(0)
    _capi.check(_capi.lib.gemm_ipc_export(full.data_ptr(), handle, ctypes.byref(offset)), "gemm_ipc_export")
    shared: List[Optional[Tuple[bytes, int]]] = [None] * world
    dist.all_gather_object(shared, (bytes(handle), offset.value), group=group)
    peers: List[Optional[int]] = []
    for r, (h, off) in enumerate(shared):
        if r == rank:
            peers.append(None)
            continue
        ptr = ctypes.c_void_p()
        _capi.check(_capi.lib.gemm_ipc_import(h, off, ctypes.byref(ptr)), "gemm_ipc_import")
        peers.append(int(ptr.value))
    return full, peers


def _mc_buffer(rows: int, N: int, device: torch.device, group) -> Tuple[torch.Tensor, int]:
    """This rank's full C for the next multicast call and the multicast address of its first element.
    Two buffers per shape, used in turn, for the reason given in ``_fused_buffer``; set up (collectively)
    on the first call for a shape."""
    key = (rows, N, device.index, _group_key(group))
    with _ipc_lock:
        entry = _mc_buffers.get(key)
    if entry is None:
        if not _equal_rows(rows, device, group):
            raise ValueError("exchange='multicast' needs equal row blocks on every rank")
        if not multicast_supported(device, group):
            raise MulticastUnavailable("NVLink multicast is not supported on every rank's GPU")
        entry = [_mc_share(rows, N, device, group), _mc_share(rows, N, device, group), 0]
        with _ipc_lock:
            _mc_buffers[key] = entry
    full, mc, _ = entry[entry[2]]
    entry[2] ^= 1
    return full, mc


def _mc_share(rows: int, N: int, device: torch.device, group) -> Tuple[torch.Tensor, int, object]:
    """A new full-size C, bound with every other rank's to one multicast object (collective)."""
    import torch.distributed._symmetric_memory as symm_mem

    world = dist.get_world_size(group)
    good, why = 0, "no multicast mapping of C"
    try:
        if symm_mem.get_backend(device) != "CUDA":
            symm_mem.set_backend("CUDA")
        full = symm_mem.empty((rows * world, N), dtype=torch.float16, device=device)
        handle = symm_mem.rendezvous(full, group if group is not None else dist.group.WORLD)
        mc = int(handle.multicast_ptr or 0)
        off = full.data_ptr() - int(handle.buffer_ptrs[handle.rank])
        good = int(mc != 0 and off >= 0 and off + full.numel() * 2 <= int(handle.buffer_size)
                   and (mc + off) % 16 == 0)
    except RuntimeError as e:   # e.g. the multicast object could not be created; every rank agrees below
        why = f"symmetric-memory set-up failed: {e}"
    flag = torch.tensor([good], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if not int(flag.item()):
        raise MulticastUnavailable(f"the symmetric-memory rendezvous gave no usable multicast mapping of C on every "
                                   f"rank ({why} on this one)" if not good else
                                   "another rank got no usable multicast mapping of C")
    return full, mc + off, handle


def _gather_cfg(rows: int, N: int, K: int) -> int:
    """The dispatched config when the fused all-gather supports it (tile_m >= 128, no split-K), else a
    CTA-pair (or, for few rows, 1-CTA) tile without split."""
    from . import _capi, dispatch

    cid = dispatch.lookup(rows, N, K)
    knobs = _capi.menu_row(cid)
    if knobs[0] >= 128 and knobs[7] == 1:
        return cid
    fallback = (256, 256, 64, 4, 2, 0, 8, 1) if rows >= 256 else (128, 128, 64, 4, 1, 0, 8, 1)
    return _capi.cfg_find(fallback)


def _fused_gather(A_local: torch.Tensor, B: torch.Tensor, M_total: Optional[int], group,
                  multicast: bool = False) -> torch.Tensor:
    from . import _capi, infinite_dreams_ext as ext

    name = "multicast" if multicast else "fused"
    if not (A_local.is_cuda and B.is_cuda):
        raise ValueError(f"exchange='{name}' needs CUDA tensors")
    ext._check_inputs(A_local, B)
    device = A_local.device
    rows, K = int(A_local.shape[0]), int(A_local.shape[1])
    N = int(B.shape[1])
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if M_total is not None and int(M_total) != rows * world:
        raise ValueError(f"row blocks sum to {rows * world}, expected {M_total}")
    if multicast and N % 8:
        raise ValueError("exchange='multicast' needs N to be a multiple of 8")
    A_local, B = A_local.contiguous(), B.contiguous()
    offset = rank * rows * N * 2
    # Both raise on unequal row blocks; the multicast one also when some rank has no multicast.
    if multicast:
        full, mc = _mc_buffer(rows, N, device, group)
    else:
        full, peers = _fused_buffer(rows, N, device, group)
        targets = [p + offset for p in peers if p is not None]
        arr = (ctypes.c_void_p * max(len(targets), 1))(*targets)
    mine = full[rank * rows:(rank + 1) * rows]
    cid = _gather_cfg(rows, N, K)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = _capi.lib.gemm_workspace_bytes(A_local.data_ptr(), B.data_ptr(), rows, N, K, K, N, cid)
        ws_ptr, ws_len = ext._workspace(device, stream, need) if need else (0, 0)
        if multicast:
            _capi.check(_capi.lib.gemm_launch_multicast(A_local.data_ptr(), B.data_ptr(), mine.data_ptr(), mc + offset,
                                                        rows, N, K, K, N, N, cid, ws_ptr or None, ws_len,
                                                        stream.cuda_stream or None), "gemm_launch_multicast")
        else:
            _capi.check(_capi.lib.gemm_launch_gather(A_local.data_ptr(), B.data_ptr(), mine.data_ptr(), rows, N, K, K,
                                                     N, N, arr, len(targets), cid, ws_ptr or None, ws_len,
                                                     stream.cuda_stream or None), "gemm_launch_gather")
        # Ordered after this rank's grid on its stream: completes once every
        # rank's grid (and so every write into this rank's C) has finished.
        done = torch.zeros(1, dtype=torch.float32, device=device)
        dist.all_reduce(done, group=group)
    return full


def release_peer_buffers(group=None) -> None:
    """Unmaps the peers' buffers and drops the fused and multicast all-gathers' own buffers.

    Collective: every rank calls it (before destroying the process group), so
    that no rank frees memory another rank still has mapped, or leaves a
    multicast object while another rank may still store through it."""
    from . import _capi

    with _ipc_lock:
        items = [(k, v) for k, v in _fused_buffers.items() if k[3] == _group_key(group)]
        mc_keys = [k for k in _mc_buffers if k[3] == _group_key(group)]
    if mc_keys:
        torch.cuda.synchronize()
        dist.barrier(group=group)   # no rank's kernel stores through a multicast address any more
        with _ipc_lock:
            for k in mc_keys:
                _mc_buffers.pop(k, None)
        torch.cuda.synchronize()
        dist.barrier(group=group)   # every rank has dropped its buffers before any goes on
    if not items:
        return
    torch.cuda.synchronize()
    for _, entry in items:
        for _, peers in entry[:2]:
            for ptr in peers:
                if ptr is not None:
                    _capi.check(_capi.lib.gemm_ipc_close(ptr), "gemm_ipc_close")
    dist.barrier(group=group)
    with _ipc_lock:
        for k, _ in items:
            _fused_buffers.pop(k, None)
