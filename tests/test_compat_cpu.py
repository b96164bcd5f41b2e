"""The reference-named custom ops (sumac_b200.compat) on the CPU: registration, fake (meta)
shapes and strides, and that a CPU call is refused like the reference's CUDA-only ops."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from sumac_b200 import compat


def test_ops_registered_under_reference_names():
    for name in ("relu_bat_c_fused", "relu_bat_c_tf32_mma_sync", "relu_bat_c_tf32_wgmma",
                 "relu_bat_reduce_fused"):
        assert hasattr(torch.ops.sumac, name)


@pytest.mark.parametrize("D", [13, 16, 17, 256])
def test_fake_shapes_and_strides(D):
    with FakeTensorMode():
        A, B, C = torch.empty(250, D), torch.empty(1000, D), torch.empty(250, D)
        assert torch.ops.sumac.relu_bat_c_fused(A, B, C, 128, 32, 1).shape == (1000, D)
        y = torch.ops.sumac.relu_bat_c_tf32_mma_sync(A, B, C, 128, 16, 2, 1)
        assert y.shape == (1000, D) and y.stride() == ((D + 7) // 8 * 8, 1)
        y = torch.ops.sumac.relu_bat_c_tf32_wgmma(A, B, C, 128, 64, 64, 16, 2, "RS")
        assert y.shape == (1000, D) and y.stride() == ((D + 7) // 8 * 8, 1)
        s1, s2 = torch.ops.sumac.relu_bat_reduce_fused(B, A, 256, 32, 1)
        assert s1.shape == (1,) and s2.shape == (1,)


def test_fake_rejects_bad_tiles_and_shapes():
    with FakeTensorMode():
        A, B, C = torch.empty(250, 16), torch.empty(1000, 16), torch.empty(250, 16)
        with pytest.raises(ValueError, match="BN must be divisible"):
            torch.ops.sumac.relu_bat_c_tf32_mma_sync(A, B, C, 128, 12, 2, 1)
        with pytest.raises(ValueError, match="num_stages"):
            torch.ops.sumac.relu_bat_c_tf32_mma_sync(A, B, C, 128, 16, 2, 4)
        with pytest.raises(RuntimeError, match="shape mismatch"):
            torch.ops.sumac.relu_bat_c_fused(A, B, torch.empty(249, 16), 128, 32, 1)


def test_cpu_tensors_are_refused():
    with pytest.raises(NotImplementedError):
        compat.relu_bat_c_fused(torch.ones(3, 2), torch.ones(4, 2), torch.ones(3, 2),
                                BM=128, BK=32, MS=1)


def test_tunable_kernel_precision_follows_config():
    from sumac_b200 import SumacConfig
    assert compat.get_tunable_kernel(SumacConfig(allow_tf32=True)).precision == 1
    assert compat.get_tunable_kernel(SumacConfig()).precision == 3
