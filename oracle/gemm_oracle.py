"""ORACLE -- test infrastructure only.  Python face of the CPU restatement.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module, and only as the checker.

* :func:`gemm_f16` -- the C restatement (``gemm_oracle.c``) of the reference
  kernel ``gemm_tiled_reg`` (src/gemm_kernels.cuh:6-83): per element an fp32
  accumulator updated in ascending k, rounded once to fp16 (RNE).
* :func:`gemm_f16_numpy` -- the same loop written with numpy (vectorised over
  the output, sequential in k), an independent restatement for small cases.
* :func:`gemm_ex` -- the same accumulation with transposed operand storage
  and the library's fused epilogue (alpha, beta * D, bias, ReLU / GELU),
  which has no reference counterpart (see gemm_oracle.c).
* :func:`tolerance` -- the acceptance bound of the build's parity tests:
  |err| <= 1e-2 * sqrt(K/1024) * max|C_ref| + 1e-3.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import List, Optional, Tuple

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_LIB_PATH = ORACLE_DIR / "_build" / "libgemm_oracle.so"
_REF_PATH = ORACLE_DIR / "_ref" / "libref_gemm.so"
_lib: Optional[ctypes.CDLL] = None


def build(reference_src: Optional[str] = None) -> None:
    """Builds the C oracle, and the reference bank when its source is given.

    ``reference_src`` (or the ``REFERENCE_SRC`` environment variable) names
    the reference's ``src/`` directory; without one, or when it holds no
    ``gemm_kernels.cuh``, only the C oracle is built."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    src = reference_src or os.environ.get("REFERENCE_SRC")
    if src and Path(src, "gemm_kernels.cuh").exists():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REFERENCE_SRC={src}"], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.oracle_gemm_f16.restype = ctypes.c_int
        lib.oracle_gemm_f16.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + [ctypes.c_int]
        lib.oracle_gemm_ex.restype = ctypes.c_int
        lib.oracle_gemm_ex.argtypes = ([ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + [ctypes.c_int] * 2 +
                                       [ctypes.c_float] * 2 + [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                                               ctypes.c_int, ctypes.c_int])
        lib.oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.oracle_f16_to_f32.restype = ctypes.c_float
        lib.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        _lib = lib
    return _lib


def _threads(n: Optional[int]) -> int:
    if n is not None:
        return max(1, int(n))
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def gemm_f16(A: np.ndarray, B: np.ndarray, threads: Optional[int] = None) -> np.ndarray:
    """C = A @ B with the reference kernel's arithmetic (fp16 in, fp16 out)."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    if A.ndim != 2 or B.ndim != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"bad shapes {A.shape} x {B.shape}")
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), dtype=np.float16)
    rc = load().oracle_gemm_f16(A.ctypes.data, B.ctypes.data, C.ctypes.data, M, N, K, K, N, N, _threads(threads))
    if rc != 0:
        raise RuntimeError(f"oracle_gemm_f16 failed ({rc})")
    return C


ACTIVATIONS = {"none": 0, "relu": 1, "gelu": 2}


def gemm_ex(A: np.ndarray, B: np.ndarray, trans_a: bool = False, trans_b: bool = False, alpha: float = 1.0,
            beta: float = 0.0, D: Optional[np.ndarray] = None, bias: Optional[np.ndarray] = None,
            activation: str = "none", threads: Optional[int] = None) -> np.ndarray:
    """act(alpha * op(A) @ op(B) + beta * D + bias) with the same accumulation as :func:`gemm_f16`.

    A and B are given as stored: A is M x K (or K x M when ``trans_a``), B is
    K x N (or N x K when ``trans_b``).  The epilogue is evaluated in fp32 and
    rounded once to fp16; D is not read when beta == 0.
    """
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    M, K = (A.shape[1], A.shape[0]) if trans_a else A.shape
    Kb, N = (B.shape[1], B.shape[0]) if trans_b else B.shape
    if K != Kb:
        raise ValueError(f"bad shapes {A.shape} (trans {trans_a}) x {B.shape} (trans {trans_b})")
    d_ptr, ldd = None, 0
    if beta != 0.0:
        D = np.ascontiguousarray(D, dtype=np.float16)
        if D.shape != (M, N):
            raise ValueError(f"D must be {(M, N)}")
        d_ptr, ldd = D.ctypes.data, N
    b_ptr = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float16).reshape(-1)
        if bias.shape != (N,):
            raise ValueError(f"bias must have {N} elements")
        b_ptr = bias.ctypes.data
    C = np.empty((M, N), dtype=np.float16)
    rc = load().oracle_gemm_ex(A.ctypes.data, B.ctypes.data, C.ctypes.data, M, N, K, A.shape[1], B.shape[1], N,
                               int(trans_a), int(trans_b), float(alpha), float(beta), d_ptr, ldd, b_ptr,
                               ACTIVATIONS[activation], _threads(threads))
    if rc != 0:
        raise RuntimeError(f"oracle_gemm_ex failed ({rc})")
    return C


def gemm_f16_numpy(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Numpy restatement of the same loop: fp32 accumulator, ascending k.

    ``a * b`` of two fp16 values is exact in fp32, so each step rounds once,
    like the reference's ``acc[i][j] += aReg[i] * bReg[j]``
    (src/gemm_kernels.cuh:61).
    """
    A32 = np.asarray(A, dtype=np.float16).astype(np.float32)
    B32 = np.asarray(B, dtype=np.float16).astype(np.float32)
    M, K = A32.shape
    acc = np.zeros((M, B32.shape[1]), dtype=np.float32)
    for k in range(K):
        acc += A32[:, k:k + 1] * B32[k:k + 1, :]
    return acc.astype(np.float16)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bit patterns through the oracle's own RNE conversion."""
    lib = load()
    flat = np.asarray(x, dtype=np.float32).ravel()
    out = np.fromiter((lib.oracle_f32_to_f16(float(v)) for v in flat), dtype=np.uint16, count=flat.size)
    return out.reshape(np.shape(x))


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    lib = load()
    flat = np.asarray(h, dtype=np.uint16).ravel()
    out = np.fromiter((lib.oracle_f16_to_f32(int(v)) for v in flat), dtype=np.float32, count=flat.size)
    return out.reshape(np.shape(h))


def tolerance(c_ref: np.ndarray, K: int) -> float:
    """|err| <= 1e-2*sqrt(K/1024)*max|C_ref| + 1e-3 (fp16 GEMM acceptance bound)."""
    mx = float(np.max(np.abs(np.asarray(c_ref, dtype=np.float32)))) if np.size(c_ref) else 0.0
    return 1e-2 * float(np.sqrt(max(K, 1) / 1024.0)) * mx + 1e-3


def load_ref() -> Optional[ctypes.CDLL]:
    """The reference kernel bank compiled from source (GPU); None if not built."""
    if not _REF_PATH.exists():
        return None
    lib = ctypes.CDLL(str(_REF_PATH))
    lib.ref_gemm_try.restype = ctypes.c_int
    lib.ref_gemm_try.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 8 + [ctypes.c_void_p]
    lib.ref_num_cfgs.restype = ctypes.c_int
    lib.ref_cfg.restype = ctypes.c_int
    lib.ref_cfg.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    return lib


def ref_cfgs(lib: ctypes.CDLL) -> List[Tuple[int, int, int, int, int]]:
    out = []
    for i in range(lib.ref_num_cfgs()):
        buf = (ctypes.c_int * 5)()
        lib.ref_cfg(i, buf)
        out.append(tuple(buf))
    return out
