"""Drop-in for the reference's compiled extension ``infinite_dreams_ext``.

The reference module (src/gemm_ext.cpp:123-132) exports three functions; the
same three names are exported here with the same argument meaning and the
same error behaviour (``RuntimeError`` with the reference's messages), backed
by the sm_100a kernel bank through its C ABI (include/gemm_sm100.h):

* ``gemm_forward(A, B, tile_m, tile_n, tile_k, stages, mma_sm=1, raster=0,
  group=8, split_k=1)`` -- explicit knobs (src/gemm_ext.cpp:57-93).  The
  reference's knobs were (tile_m, tile_n, tile_k, tm, tn); the register
  micro-tile (tm, tn) has no meaning for tcgen05, so the positions after
  tile_k carry the Blackwell knobs.  A tuple that is not in the menu raises
  (the reference returned an uninitialised tensor, gemm_ext.cpp:35 + F7).
* ``gemm_forward_cfg(A, B, cfg_id)`` -- menu id (src/gemm_ext.cpp:95-106).
* ``gemm_cfg_table_cpu()`` -- the menu as a CPU int32 tensor
  ``[num_cfg, len(CFG_COLUMNS)]`` (src/gemm_ext.cpp:108-120).

``gemm_ex`` goes beyond the reference: transposed operand views read in
place and a fused epilogue (alpha, beta * C, bias, ReLU / GELU).

Like the reference, inputs are made contiguous, C is allocated from torch's
caching allocator on A's device, and the launch is asynchronous on the
current stream.  Split-K / repacking workspace is cached per (device, stream)
and zero-initialised once, as the C ABI requires.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional, Tuple

import torch

from . import _capi
from ._capi import GemmError, lib

CFG_COLUMNS: Tuple[str, ...] = tuple(_capi.menu()[0])
NUM_CFG: int = int(lib.gemm_num_cfgs())

# The compiled torch binding of the same C ABI (csrc/torch_ext.cpp) takes the
# per-call Python work off small launches; the ctypes path below remains for
# builds without it (INFINITE_DREAMS_NO_TORCH_EXT=1 selects it explicitly).
_fast = None
if not os.environ.get("INFINITE_DREAMS_NO_TORCH_EXT"):
    try:
        from . import _torch_ext as _fast  # type: ignore[no-redef]
    except ImportError:
        _fast = None

_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> Tuple[int, int]:
    if nbytes == 0:
        return 0, 0
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            # Grow geometrically; zeros satisfies the "ticket region is zero" contract.
            size = max(nbytes, 0 if ws is None else 2 * ws.numel())
            with torch.cuda.stream(stream):
                ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws.data_ptr(), ws.numel()


def reset_workspaces() -> None:
    """Drops cached workspaces (needed after a device-side timeout)."""
    with _ws_lock:
        _workspaces.clear()
    if _fast is not None:
        _fast.reset_workspaces()


def _check_inputs(A: torch.Tensor, B: torch.Tensor) -> None:
    # Same checks and messages as src/gemm_ext.cpp:66-73,86.
    if not isinstance(A, torch.Tensor) or not A.is_cuda:
        raise RuntimeError("A must be CUDA tensor")
    if not isinstance(B, torch.Tensor) or not B.is_cuda:
        raise RuntimeError("B must be CUDA tensor")
    if A.dtype != torch.float16:
        raise RuntimeError("A must be float16")
    if B.dtype != torch.float16:
        raise RuntimeError("B must be float16")
    if A.dim() != 2:
        raise RuntimeError("A must be 2D (M x K)")
    if B.dim() != 2:
        raise RuntimeError("B must be 2D (K x N)")
    if A.size(1) != B.size(0):
        raise RuntimeError("Inner dimensions must match: A is (M x K), B is (K x N)")
    if A.get_device() != B.get_device():
        raise RuntimeError("A and B must be on the same CUDA device")


def _launch(A: torch.Tensor, B: torch.Tensor, cfg_id: int, out: Optional[torch.Tensor]) -> torch.Tensor:
    if A.get_device() != torch.cuda.current_device():
        with torch.cuda.device(A.device):
            return _launch_here(A, B, cfg_id, out)
    return _launch_here(A, B, cfg_id, out)


def _launch_here(A: torch.Tensor, B: torch.Tensor, cfg_id: int, out: Optional[torch.Tensor]) -> torch.Tensor:
    """Launch on A's device, which is the current device."""
    M, K = A.shape
    N = B.shape[1]
    dev = A.device
    A = A.contiguous()
    B = B.contiguous()
    if out is None:
        C = torch.empty((M, N), dtype=torch.float16, device=dev)
    else:
        if (out.dtype != torch.float16 or out.shape != (M, N) or out.device != dev
                or not out.is_contiguous()):
            raise RuntimeError("out must be a contiguous float16 (M x N) tensor on A's device")
        C = out
    stream = torch.cuda.current_stream(dev)
    a_ptr, b_ptr = A.data_ptr(), B.data_ptr()
    need = lib.gemm_workspace_bytes(a_ptr, b_ptr, M, N, K, K, N, cfg_id)
    ws_ptr, ws_len = _workspace(dev, stream, need) if need else (0, 0)
    st = lib.gemm_launch(a_ptr, b_ptr, C.data_ptr(), M, N, K, K, N, N, cfg_id,
                         ws_ptr or None, ws_len, stream.cuda_stream or None)
    if st:
        _capi.check(st, "gemm_launch")
    return C


def gemm_forward(A: torch.Tensor, B: torch.Tensor, tile_m: int, tile_n: int, tile_k: int, stages: int,
                 mma_sm: int = 1, raster: int = 0, group: int = 8, split_k: int = 1,
                 *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FP16 GEMM forward (CUDA) with explicit knobs; the tuple must be in the menu."""
    _check_inputs(A, B)
    if tile_m <= 0 or tile_n <= 0 or tile_k <= 0:
        raise RuntimeError("tile_m/tile_n/tile_k must be > 0")
    if stages <= 0 or mma_sm <= 0 or group <= 0 or split_k <= 0:
        raise RuntimeError("stages/mma_sm/group/split_k must be > 0")
    knobs = (tile_m, tile_n, tile_k, stages, mma_sm, raster, group, split_k)
    cfg_id = _capi.cfg_find(knobs)
    if cfg_id < 0:
        raise RuntimeError(f"knob tuple {knobs} is not in the kernel bank menu "
                           f"(columns {', '.join(CFG_COLUMNS)})")
    if _fast is not None:
        return _fast.gemm_forward_cfg(A, B, cfg_id, out)
    return _launch(A, B, cfg_id, out)


def gemm_forward_cfg(A: torch.Tensor, B: torch.Tensor, cfg_id: int, *,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FP16 GEMM forward (CUDA) using cfg_id from the static menu."""
    if cfg_id < 0:
        raise RuntimeError("cfg_id must be >= 0")
    if cfg_id >= NUM_CFG:
        raise RuntimeError("cfg_id out of range")
    if _fast is not None:
        return _fast.gemm_forward_cfg(A, B, int(cfg_id), out)
    _check_inputs(A, B)
    return _launch(A, B, int(cfg_id), out)


def _operand(X: torch.Tensor) -> Tuple[torch.Tensor, int, int]:
    """(tensor, trans, pitch) for a logical [R, C] operand read in place.

    A row-major view (unit column stride) is passed as stored; a transposed
    view (unit row stride, e.g. ``W.t()``) is passed as its K-major storage
    with trans = 1, which the kernels read without a copy.  Anything else is
    made contiguous first.
    """
    R, C = X.shape
    s0, s1 = X.stride()
    if (s1 == 1 or C <= 1) and s0 >= max(C, 1):
        return X, 0, s0
    if (s0 == 1 or R <= 1) and s1 >= max(R, 1):
        return X, 1, s1
    X = X.contiguous()
    return X, 0, max(C, 1)


def gemm_ex(A: torch.Tensor, B: torch.Tensor, *, alpha: float = 1.0, beta: float = 0.0,
            C: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None, activation: str = "none",
            cfg_id: Optional[int] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = act(alpha * A @ B + beta * C + bias), fp16, fused into the GEMM's epilogue.

    A is a logical [M, K] and B a logical [K, N] fp16 CUDA tensor; row-major
    and transposed views (``x.t()``) are read in place (gemm_launch_ex's
    trans flags), other strides are copied.  C ([M, N], read only when
    beta != 0) may be ``out`` itself for an in-place update; bias is [N].
    activation: "none", "relu" or "gelu" (erf form).  cfg_id defaults to the
    per-shape dispatch table entry, else the heuristic.
    """
    _check_inputs(A, B)
    if activation not in _capi.ACTIVATIONS:
        raise RuntimeError(f"activation must be one of {sorted(_capi.ACTIVATIONS)}")
    M, K = A.shape
    N = B.shape[1]
    dev = A.device
    if _fast is not None:
        if cfg_id is None:
            from . import dispatch
            cfg_id = dispatch.lookup(M, N, K, epilogue=(beta != 0.0 or activation != "none"))
        return _fast.gemm_ex(A, B, int(cfg_id), float(alpha), float(beta), C, bias, _capi.ACTIVATIONS[activation],
                             out)
    if beta != 0.0:
        if C is None:
            raise RuntimeError("beta != 0 needs C")
        if C.dtype != torch.float16 or tuple(C.shape) != (M, N) or C.device != dev:
            raise RuntimeError("C must be a float16 (M x N) tensor on A's device")
        if C.stride(1) != 1 and N > 1:
            C = C.contiguous()
    if bias is not None:
        if bias.dtype != torch.float16 or bias.numel() != N or bias.device != dev:
            raise RuntimeError("bias must be a float16 tensor of N elements on A's device")
        bias = bias.reshape(N).contiguous()
    if cfg_id is None:
        from . import dispatch
        cfg_id = dispatch.lookup(M, N, K, epilogue=(beta != 0.0 or activation != "none"))
    elif not 0 <= int(cfg_id) < NUM_CFG:
        raise RuntimeError("cfg_id out of range")
    with torch.cuda.device(dev):
        A_s, ta, lda = _operand(A)
        B_s, tb, ldb = _operand(B)
        if out is None:
            out = torch.empty((M, N), dtype=torch.float16, device=dev)
        elif (out.dtype != torch.float16 or tuple(out.shape) != (M, N) or out.device != dev
              or (out.stride(1) != 1 and N > 1)):
            raise RuntimeError("out must be a float16 (M x N) tensor with unit column stride on A's device")
        stream = torch.cuda.current_stream(dev)
        a_ptr, b_ptr = A_s.data_ptr(), B_s.data_ptr()
        need = lib.gemm_workspace_bytes_ex(a_ptr, b_ptr, M, N, K, lda, ldb, ta, tb, int(cfg_id))
        ws_ptr, ws_len = _workspace(dev, stream, need) if need else (0, 0)
        d_ptr, ldd = (C.data_ptr(), max(C.stride(0), N)) if beta != 0.0 else (None, 0)
        st = lib.gemm_launch_ex(a_ptr, b_ptr, out.data_ptr(), M, N, K, lda, ldb, max(out.stride(0), N), ta, tb,
                                float(alpha), float(beta), d_ptr, ldd,
                                bias.data_ptr() if bias is not None else None, _capi.ACTIVATIONS[activation],
                                int(cfg_id), ws_ptr or None, ws_len, stream.cuda_stream or None)
        if st:
            _capi.check(st, "gemm_launch_ex")
    return out


def gemm_cfg_table_cpu() -> torch.Tensor:
    """CPU int32 tensor [num_cfg, len(CFG_COLUMNS)], columns CFG_COLUMNS."""
    cols, rows = _capi.menu()
    return torch.tensor(rows, dtype=torch.int32).reshape(len(rows), len(cols))


def default_cfg(M: int, N: int, K: int) -> int:
    return int(lib.gemm_default_cfg(M, N, K))


def check_device_errors(device: Optional[int] = None) -> None:
    """Raises if a kernel on `device` gave up on a bounded wait (synchronises)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    code = ctypes.c_int(0)
    st = lib.gemm_device_error(dev, ctypes.byref(code))
    if st != _capi.GEMM_OK:
        reset_workspaces()
        raise GemmError(st, f"device {dev}: kernel error bits {code.value}")


__all__ = ["gemm_forward", "gemm_forward_cfg", "gemm_ex", "gemm_cfg_table_cpu", "CFG_COLUMNS", "NUM_CFG",
           "default_cfg", "check_device_errors", "GemmError", "reset_workspaces"]
