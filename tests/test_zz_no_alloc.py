"""sumac_relu_bat_reduce_noalloc through the C ABI.

This entry point serves callers that cannot give the library device memory: hosts whose own
allocator owns the GPU (a MATLAB gpuArray binding, a serving process that reserved the device) or
paths that must not call cudaMalloc / cudaFree because those can synchronise the device. It keeps
its scratch in a fixed device array of the library, so the check here is that two calls in a row
give the same sums as the regular, workspace-taking sumac_relu_bat_reduce, and that a problem too
large for the fixed scratch is refused with a clear error. This file is collected last on purpose.
"""

import numpy as np
import pytest
import torch

from sumac_b200 import _native

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the 3xTF32 tolerance of the kernel parity tests


def _regular(lib, A, B, D, prec):
    M, N = A.shape[0], B.shape[0]
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    nb = lib.sumac_relu_bat_reduce_workspace_bytes(M, N, D, prec)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sumac_relu_bat_reduce(A.data_ptr(), B.data_ptr(), M, N, D, out.data_ptr(), prec,
                                   ws.data_ptr(), nb, err.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sumac_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


def _noalloc(lib, A, B, D, prec):
    M, N = A.shape[0], B.shape[0]
    out = torch.full((2,), -1.0, dtype=torch.float64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sumac_relu_bat_reduce_noalloc(A.data_ptr(), B.data_ptr(), M, N, D, out.data_ptr(),
                                           prec, err.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sumac_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("prec", [_native.SUMAC_3XTF32, _native.SUMAC_TF32])
def test_noalloc_matches_regular_entry_point_twice(prec):
    lib = _native.lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    D = 16
    inputs = [(torch.randn(20000, D, device="cuda", generator=g),
               torch.randn(250, D, device="cuda", generator=g)),
              (torch.randn(7000, D, device="cuda", generator=g),
               torch.randn(1300, D, device="cuda", generator=g))]
    for A, B in inputs:  # two calls in a row share (and reuse) the fixed scratch
        got = _noalloc(lib, A, B, D, prec)
        want = _regular(lib, A, B, D, prec)
        np.testing.assert_allclose(got, want, rtol=RTOL)


def test_noalloc_rejects_problem_larger_than_scratch():
    lib = _native.lib()
    cap = lib.sumac_noalloc_scratch_bytes()
    M = cap // (16 * 4) + 1  # the padded copy of A alone exceeds the scratch
    A = torch.empty((M, 16), device="cuda")
    B = torch.empty((8, 16), device="cuda")
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sumac_relu_bat_reduce_noalloc(A.data_ptr(), B.data_ptr(), M, 8, 16, out.data_ptr(),
                                           _native.SUMAC_3XTF32, err.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == -3
    assert b"fixed scratch" in lib.sumac_last_error()


@pytest.mark.parametrize("M,N,D", [(-5, 8, 16), (100, -1, 16), (100, 8, 0)])
def test_noalloc_rejects_bad_shapes_as_argument_errors(M, N, D):
    lib = _native.lib()
    A = torch.empty((8, 16), device="cuda")
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sumac_relu_bat_reduce_noalloc(A.data_ptr(), A.data_ptr(), M, N, D, out.data_ptr(),
                                           _native.SUMAC_3XTF32, err.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == -1  # SUMAC_ERR_ARG, not the scratch-size error
