"""Pins the oracle against the reference kernel itself (GPU).

oracle/_ref/libref_gemm.so is the reference's gemm_tiled_reg
(src/gemm_kernels.cuh:6-83) compiled from its own source by oracle/Makefile.
Its output must equal the CPU oracle bit for bit for every instantiated tile
configuration: the oracle restates the kernel's arithmetic exactly.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import make_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_lib(cuda_device):
    lib = oracle.load_ref()
    if lib is None:
        pytest.skip("reference bank not built (oracle/_ref missing)")
    return lib


def _ref_run(lib, A, B, cfg):
    M, K = A.shape
    N = B.shape[1]
    Ad, Bd = A.cuda(), B.cuda()
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.ref_gemm_try(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K, *cfg,
                          torch.cuda.current_stream().cuda_stream or None)
    assert rc == 1, f"reference bank did not launch {cfg} (rc {rc})"
    torch.cuda.synchronize()
    return C.cpu().numpy()


@pytest.mark.parametrize("M,N,K,dist", [(512, 512, 512, "uniform"), (1000, 3000, 777, "uniform"),
                                        (7, 12288, 96, "uniform"), (64, 4096, 4096, "skinny"),
                                        (129, 65, 1, "uniform"), (33, 257, 1025, "uniform")])
def test_reference_kernel_equals_oracle(ref_lib, M, N, K, dist):
    A, B = make_inputs(M, N, K, dist, seed=M + N + K)
    exp = oracle.gemm_f16(A.numpy(), B.numpy())
    for cfg in oracle.ref_cfgs(ref_lib):
        got = _ref_run(ref_lib, A, B, cfg)
        assert np.array_equal(got.view(np.uint16), exp.view(np.uint16)), f"{M}x{N}x{K} cfg {cfg}"
