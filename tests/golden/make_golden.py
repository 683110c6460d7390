"""Generates tests/golden/ref_gemm_golden.npz from the reference kernel itself.

Run on a B200 after `make -C oracle ref REFERENCE_SRC=<reference src/>` (which compiles the reference's
src/gemm_kernels.cuh for sm_100a into oracle/_ref/libref_gemm.so):

    python tests/golden/make_golden.py

For every case below, the seeded fp16 inputs A, B are multiplied by EVERY
tile configuration instantiated in the reference bank; the outputs must agree
with each other (the reference's arithmetic does not depend on the tile) and
the first one is stored.  tests/test_oracle_cpu.py then checks the CPU oracle
against these outputs bit for bit, without a GPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def cases():
    """(name, A, B) with small shapes and edge-case values."""
    rng = np.random.default_rng(20250225)
    out = []

    def uni(m, k, n, scale=1.0):
        return (rng.uniform(-1, 1, (m, k)) * scale).astype(np.float16), (rng.uniform(-1, 1, (k, n)) * scale).astype(np.float16)

    for (m, n, k) in [(1, 1, 1), (3, 5, 7), (16, 16, 16), (33, 65, 129), (128, 64, 200), (5, 300, 64)]:
        A, B = uni(m, k, n)
        out.append((f"uniform_{m}x{n}x{k}", A, B))
    A = rng.standard_normal((17, 300)).astype(np.float16)
    B = (rng.standard_normal((300, 40)) * 0.02).astype(np.float16)
    out.append(("skinny_17x40x300", A, B))
    # overflow to +-inf in the fp16 output, and products near fp16 max
    A, B = uni(8, 16, 24, 300.0)
    out.append(("overflow_8x24x16", A, B))
    # tiny magnitudes: fp16 subnormal inputs and outputs
    A, B = uni(8, 32, 24, 1e-3)
    A[0, :8] = np.float16(6e-8)
    out.append(("subnormal_8x24x32", A, B))
    # cancellation: rows that sum to exact zero, and signed zeros
    A = np.zeros((4, 8), np.float16)
    A[0] = [1, -1, 2, -2, 0.5, -0.5, 0, -0.0]
    A[1] = -0.0
    B = np.ones((8, 6), np.float16)
    B[:, 3] = -1
    out.append(("cancel_4x6x8", A, B))
    return out


def main() -> None:
    import torch

    import oracle

    lib = oracle.load_ref()
    if lib is None:
        raise SystemExit("oracle/_ref/libref_gemm.so is missing: run `make -C oracle ref REFERENCE_SRC=<reference src/>` first")
    cfgs = oracle.ref_cfgs(lib)
    arrays = {}
    names = []
    for name, A, B in cases():
        M, K = A.shape
        N = B.shape[1]
        outs = []
        for cfg in cfgs:
            Ad = torch.from_numpy(A).cuda()
            Bd = torch.from_numpy(B).cuda()
            C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            rc = lib.ref_gemm_try(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K, *cfg,
                                  torch.cuda.current_stream().cuda_stream or None)
            assert rc == 1, (name, cfg, rc)
            torch.cuda.synchronize()
            outs.append(C.cpu().numpy().view(np.uint16))
        for o in outs[1:]:
            assert np.array_equal(o, outs[0]), f"{name}: reference output depends on the tile config"
        arrays[f"{name}__A"] = A.view(np.uint16)
        arrays[f"{name}__B"] = B.view(np.uint16)
        arrays[f"{name}__C"] = outs[0]
        names.append(name)
    arrays["cases"] = np.array(names)
    arrays["ref_cfgs"] = np.array(cfgs, dtype=np.int32)
    out = Path(__file__).resolve().parent / "ref_gemm_golden.npz"
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({len(names)} cases x {len(cfgs)} reference configs, all configs agree)")


if __name__ == "__main__":
    main()
