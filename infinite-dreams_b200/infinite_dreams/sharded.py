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

Only NCCL moves remote data: no kernel here reads another GPU's memory.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

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
                 chunks: int = 1) -> torch.Tensor:
    """This rank's rows of C = A @ B (or all of C when gather=True).

    A_local holds this rank's row block (``row_block``); B is the full
    replicated K x N operand.  ``compute`` defaults to the dispatched
    kernel-bank GEMM.  ``chunks`` > 1 overlaps the all-gather with the
    compute (equal row blocks only; other cases fall back to one exchange).
    """
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
