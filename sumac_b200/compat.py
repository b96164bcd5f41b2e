"""The reference's operator boundary, served by this library's kernels.

Importing this module registers, under the reference's own names and signatures, the torch
custom ops that the reference registers in ``src/sumac/kernels/*/custom_op.py``, so that code
written against those ops (the reference's kernel tests and ``kernel_benchmarks/``) runs on the
sm_100a kernels unchanged:

* ``sumac::relu_bat_c_fused(A, B, C, BM, BK, MS) -> Y[M, D]`` — fp32 relu_bat_c
  (``relu_batc_jit/custom_op.py:7-42``); served by the 3xTF32 (fp32-accurate) product.
* ``sumac::relu_bat_c_tf32_mma_sync(A, B, C, BM, BN, M_TILES, num_stages)`` — TF32 relu_bat_c
  returning an ``(M, D)`` view with row stride ``round_up(D, 8)``
  (``relu_batc_tf32_jit/custom_op.py:33-79``); served by the TF32 product.
* ``sumac::relu_bat_c_tf32_wgmma(A, B, C, BM, BN, WGMMA_S_N, WGMMA_Y_N, num_stages,
  wgmma_mode)`` — the reference's Hopper-only TF32 op (``:82-145``); the same TF32 product.
* ``sumac::relu_bat_reduce_fused(A, B, BM, BK, MS) -> (sum ReLU(A B^T), sum ReLU(A B^T)^2)`` as
  float32 ``[1]`` tensors (``relu_bat_reduce_jit/custom_op.py:7-32``, ``jit_kernel.py:112-132``),
  with autograd (``custom_op.py:34-91``). The backward never forms the M x N matrix: each
  gradient is one fused product pass, ``ReLU(A B^T) B`` and ``ReLU(A B^T)^T A`` for the sum of
  squares, ``step(A B^T) B`` and ``step(A B^T)^T A`` for the sum.

The tile parameters (BM, BK, MS, BN, ...) are validated as the reference validates them and
otherwise ignored: the kernels here choose their own tiles per rank. Every op requires CUDA float32
tensors; there is no CPU path (the reference's ops are registered for ``device_types="cuda"``
only). ``get_tunable_kernel`` and ``AutotuneReluBatReduce`` stand in for the reference's autotuner
objects (``kernels/tuning/relu_bat_c/__init__.py:49-78``, ``tuning/relu_bat_reduce``): callables
taking the same ``(A, B, C)`` / ``(A, B)`` tuples, with a no-op ``resolve_decision``.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import ops
from ._native import SUMAC_3XTF32, SUMAC_TF32


def _round_up(value: int, multiple: int) -> int:
    return ((value + multiple - 1) // multiple) * multiple


# ------------------------------------------------------------------ argument checks
def _check_fused(A: Tensor, B: Tensor, C: Tensor) -> None:
    """The checks and messages of relu_batc_jit/jit_kernel.py:99-117."""
    if not (A.is_cuda and B.is_cuda and C.is_cuda):
        raise ValueError("A, B, and C must be CUDA tensors")
    if not (A.dtype == B.dtype == C.dtype == torch.float32):
        raise ValueError("A, B, and C must be float32")
    if not (A.is_contiguous() and B.is_contiguous() and C.is_contiguous()):
        raise ValueError("A, B, and C must be contiguous")
    if not (A.ndim == B.ndim == C.ndim == 2):
        raise ValueError("A, B, and C must be 2D")
    N, D = A.shape
    if B.shape[1] != D:
        raise ValueError(f"B.shape[1] must equal A.shape[1], got {B.shape[1]} vs {D}")
    if tuple(C.shape) != (N, D):
        raise ValueError(f"C must have shape {(N, D)}, got {tuple(C.shape)}")


def _check_tf32(A: Tensor, B: Tensor, C: Tensor) -> None:
    """The shape / dtype checks of relu_batc_tf32_jit/jit_kernel_tf32_sync.py:230-250."""
    if not (A.is_cuda and B.is_cuda and C.is_cuda):
        raise ValueError("A, B, and C must be CUDA tensors")
    if not (A.device == B.device == C.device):
        raise ValueError("A, B, and C must be on the same CUDA device")
    if A.dtype != torch.float32 or B.dtype != torch.float32 or C.dtype != torch.float32:
        raise ValueError("A, B, and C must be float32 tensors")
    if not (A.is_contiguous() and B.is_contiguous() and C.is_contiguous()):
        raise ValueError("A, B, and C must be contiguous")
    if A.ndim != 2 or B.ndim != 2 or C.ndim != 2:
        raise ValueError("A, B, and C must be rank-2 tensors")
    N, D = A.shape
    if B.shape[1] != D:
        raise ValueError(f"B has D={B.shape[1]}, expected {D}")
    if tuple(C.shape) != (N, D):
        raise ValueError(f"C must have shape [{N}, {D}], got {tuple(C.shape)}")
    if D < 1:
        raise ValueError("D must be >= 1")


def _check_mma_sync_tiles(BM: int, BN: int, M_TILES: int, num_stages: int) -> None:
    if BN % 8 != 0:
        raise ValueError("BN must be divisible by MMA_N=8")
    if num_stages < 1 or num_stages > 3:
        raise ValueError("num_stages must be in [1, 3]")
    if M_TILES < 1 or BM % (M_TILES * 16) != 0:
        raise ValueError("BM must be divisible by M_TILES * 16")


def _check_wgmma_tiles(BM: int, BN: int, S_N: int, Y_N: int, num_stages: int, mode: str) -> None:
    if S_N not in (16, 32, 64, 128):
        raise ValueError("WGMMA_S_N must be one of 16, 32, 64, or 128")
    if Y_N not in (16, 32, 64, 128):
        raise ValueError("WGMMA_Y_N must be one of 16, 32, 64, or 128")
    if BN % S_N != 0:
        raise ValueError("BN must be divisible by WGMMA_S_N")
    if num_stages not in (1, 2, 3):
        raise ValueError("num_stages must be 1, 2, or 3")
    if str(mode).upper() not in ("RS", "SS"):
        raise ValueError("wgmma_mode must be 'RS' or 'SS'")
    if BM % 64 != 0:
        raise ValueError("BM must be divisible by 64")


def _check_reduce(A: Tensor, B: Tensor) -> None:
    """The checks and messages of relu_bat_reduce_jit/jit_kernel.py:94-106."""
    if not (A.is_cuda and B.is_cuda):
        raise ValueError("A and B must be CUDA tensors")
    if not (A.dtype == B.dtype == torch.float32):
        raise ValueError("A and B must be float32")
    if not (A.is_contiguous() and B.is_contiguous()):
        raise ValueError("A and B must be contiguous")
    if not (A.ndim == B.ndim == 2):
        raise ValueError("A and B must be 2D")
    if A.shape[1] != B.shape[1]:
        raise ValueError(f"Inner dimensions must match, got {A.shape[1]} and {B.shape[1]}")


def _fake_shapes(A: Tensor, B: Tensor, C: Tensor) -> tuple[int, int]:
    if A.dim() != 2 or B.dim() != 2 or C.dim() != 2:
        raise RuntimeError("expected 2D tensors")
    N, D = A.shape
    M, DB = B.shape
    if DB != D or tuple(C.shape) != (N, D):
        raise RuntimeError("shape mismatch")
    return M, D


def _tf32_strided(A: Tensor, B: Tensor, C: Tensor) -> Tensor:
    """TF32 relu_bat_c returned as the reference's TF32 ops return it: an (M, D) view of an
    (M, round_up(D, 8)) buffer."""
    M, D = B.shape[0], A.shape[1]
    out = torch.empty((M, _round_up(D, 8)), dtype=torch.float32, device=A.device)
    out[:, :D] = ops.relu_bat_c(A, B, C, SUMAC_TF32)
    return out[:, :D]


# ------------------------------------------------------------------ sumac::relu_bat_c_fused
@torch.library.custom_op("sumac::relu_bat_c_fused", mutates_args=(), device_types="cuda")
def relu_bat_c_fused_op(A: Tensor, B: Tensor, C: Tensor, BM: int, BK: int, MS: int) -> Tensor:
    _check_fused(A, B, C)
    return ops.relu_bat_c(A, B, C, SUMAC_3XTF32)


@relu_bat_c_fused_op.register_fake
def _(A, B, C, BM, BK, MS):
    M, D = _fake_shapes(A, B, C)
    return A.new_empty((M, D))


# ------------------------------------------------------------------ sumac::relu_bat_c_tf32_*
@torch.library.custom_op("sumac::relu_bat_c_tf32_mma_sync", mutates_args=(), device_types="cuda")
def relu_bat_c_tf32_mma_sync_op(A: Tensor, B: Tensor, C: Tensor, BM: int, BN: int, M_TILES: int,
                                num_stages: int) -> Tensor:
    _check_tf32(A, B, C)
    _check_mma_sync_tiles(BM, BN, M_TILES, num_stages)
    return _tf32_strided(A, B, C)


@relu_bat_c_tf32_mma_sync_op.register_fake
def _(A, B, C, BM, BN, M_TILES, num_stages):
    M, D = _fake_shapes(A, B, C)
    _check_mma_sync_tiles(BM, BN, M_TILES, num_stages)
    return A.new_empty_strided((M, D), (_round_up(D, 8), 1))


@torch.library.custom_op("sumac::relu_bat_c_tf32_wgmma", mutates_args=(), device_types="cuda")
def relu_bat_c_tf32_wgmma_op(A: Tensor, B: Tensor, C: Tensor, BM: int, BN: int, WGMMA_S_N: int,
                             WGMMA_Y_N: int, num_stages: int, wgmma_mode: str) -> Tensor:
    _check_tf32(A, B, C)
    _check_wgmma_tiles(BM, BN, WGMMA_S_N, WGMMA_Y_N, num_stages, wgmma_mode)
    return _tf32_strided(A, B, C)


@relu_bat_c_tf32_wgmma_op.register_fake
def _(A, B, C, BM, BN, WGMMA_S_N, WGMMA_Y_N, num_stages, wgmma_mode):
    M, D = _fake_shapes(A, B, C)
    _check_wgmma_tiles(BM, BN, WGMMA_S_N, WGMMA_Y_N, num_stages, wgmma_mode)
    return A.new_empty_strided((M, D), (_round_up(D, 8), 1))


# ------------------------------------------------------------------ sumac::relu_bat_reduce_fused
@torch.library.custom_op("sumac::relu_bat_reduce_fused", mutates_args=(), device_types="cuda")
def relu_bat_reduce_fused_op(A: Tensor, B: Tensor, BM: int, BK: int,
                             MS: int) -> tuple[Tensor, Tensor]:
    _check_reduce(A, B)
    out = ops.relu_bat_reduce(A, B, SUMAC_3XTF32)
    # the reference accumulates in float64 and returns float32 [1] tensors (jit_kernel.py:132)
    return out[0:1].float(), out[1:2].float()


@relu_bat_reduce_fused_op.register_fake
def _(A, B, BM, BK, MS):
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("expected 2D tensors")
    if A.shape[1] != B.shape[1]:
        raise RuntimeError("shape mismatch")
    return A.new_empty((1,)), A.new_empty((1,))


def _reduce_setup_context(ctx, inputs, output) -> None:
    A, B = inputs[:2]
    ctx.save_for_backward(A, B)


def _reduce_backward(ctx, grad_sum_sr, grad_sum_sr2):
    """d/dA sum ReLU(A B^T)^2 = 2 ReLU(A B^T) B and d/dB = 2 ReLU(A B^T)^T A; d/dA sum ReLU(A B^T)
    = step(A B^T) B and d/dB = step(A B^T)^T A (custom_op.py:39-85). Each product is one fused
    pass (relu_bat_c(F, X, C) = map(X F^T) C), fp32-accurate."""
    A, B = ctx.saved_tensors
    need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    A = A.contiguous()
    B = B.contiguous()
    grad_A = grad_B = None

    def add(acc, term):
        return term if acc is None else acc + term

    if grad_sum_sr2 is not None:
        scale = 2.0 * grad_sum_sr2.to(A.dtype)
        if need_a:
            grad_A = add(grad_A, scale * ops.relu_bat_c(B, A, B, SUMAC_3XTF32))
        if need_b:
            grad_B = add(grad_B, scale * ops.relu_bat_c(A, B, A, SUMAC_3XTF32))
    if grad_sum_sr is not None and (need_a or need_b):
        g = grad_sum_sr.to(A.dtype)
        if need_a:
            grad_A = add(grad_A, g * ops.relu_bat_c(B, A, B, SUMAC_3XTF32, ops.SUMAC_STEP))
        if need_b:
            grad_B = add(grad_B, g * ops.relu_bat_c(A, B, A, SUMAC_3XTF32, ops.SUMAC_STEP))
    return grad_A, grad_B, None, None, None


relu_bat_reduce_fused_op.register_autograd(_reduce_backward, setup_context=_reduce_setup_context)


# ------------------------------------------------------------------ the reference's api.py names
def relu_bat_c_fused(A: Tensor, B: Tensor, C: Tensor, *, BM: int, BK: int, MS: int) -> Tensor:
    """relu_batc_jit/api.py: Y = ReLU(B A^T) C in fp32."""
    return relu_bat_c_fused_op(A, B, C, BM, BK, MS)


def relu_bat_c_tf32_mma_sync(A: Tensor, B: Tensor, C: Tensor, *, BM: int, BN: int, M_TILES: int,
                             num_stages: int = 2) -> Tensor:
    """relu_batc_tf32_jit/api.py: Y = ReLU(B A^T) C in TF32."""
    return relu_bat_c_tf32_mma_sync_op(A, B, C, BM, BN, M_TILES, num_stages)


def relu_bat_c_tf32_wgmma(A: Tensor, B: Tensor, C: Tensor, *, BM: int, BN: int, WGMMA_N: int = 16,
                          WGMMA_S_N: int | None = None, WGMMA_Y_N: int | None = None,
                          num_stages: int = 2, wgmma_mode: str = "RS") -> Tensor:
    """relu_batc_tf32_jit/api.py: the Hopper op's signature, served by the TF32 product."""
    S_N = WGMMA_N if WGMMA_S_N is None else WGMMA_S_N
    Y_N = WGMMA_N if WGMMA_Y_N is None else WGMMA_Y_N
    mode = str(wgmma_mode).upper()
    if mode not in ("RS", "SS"):
        raise ValueError("wgmma_mode must be 'RS' or 'SS'")
    return relu_bat_c_tf32_wgmma_op(A, B, C, BM, BN, S_N, Y_N, num_stages, mode)


def relu_bat_reduce_fused(A: Tensor, B: Tensor, BM: int, BK: int, MS: int) -> tuple[Tensor, Tensor]:
    """relu_bat_reduce_jit/api.py: (sum ReLU(A B^T), sum ReLU(A B^T)^2) as float32 [1] tensors."""
    return relu_bat_reduce_fused_op(A, B, BM, BK, MS)


# ------------------------------------------------------------------ autotuner stand-ins
class ReluBatCKernel:
    """What ``get_tunable_kernel(cfg)`` returns: ``kernel((A, B, C))`` = ReLU(B A^T) C at the
    precision ``cfg.allow_tf32`` selects (3xTF32 for the fp32 default, TF32 otherwise)."""

    def __init__(self, allow_tf32: bool):
        self.precision = SUMAC_TF32 if allow_tf32 else SUMAC_3XTF32

    def resolve_decision(self, params) -> None:
        """Kernel tiles are fixed per rank here: nothing to decide."""

    def __call__(self, params) -> Tensor:
        A, B, C = params
        return ops.relu_bat_c(A.contiguous(), B.contiguous(), C.contiguous(), self.precision)


def get_tunable_kernel(cfg) -> ReluBatCKernel:
    """Stand-in for kernels/tuning/relu_bat_c/__init__.py:49-78."""
    return ReluBatCKernel(bool(getattr(cfg, "allow_tf32", False)))


class AutotuneReluBatReduce:
    """Stand-in for kernels/tuning/relu_bat_reduce: ``kernel((A, B))`` = the reduce op (with
    autograd), fp32-accurate."""

    def __init__(self, *args, **kwargs):
        pass

    def resolve_decision(self, params) -> None:
        pass

    def __call__(self, params) -> tuple[Tensor, Tensor]:
        A, B = params
        return relu_bat_reduce_fused_op(A.contiguous(), B.contiguous(), 0, 0, 0)
