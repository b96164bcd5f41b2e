"""Public entry point with the reference's signature and behaviour (src/sumac/sumac.py:18-88)."""
from __future__ import annotations

import warnings
from contextlib import contextmanager

import torch
from torch import Tensor

from .config import SumacConfig, SumacMethod
from .data import prune_zero_rows_cols, restore_zero_rows_cols
from .validation import validate_sumac_inputs


@contextmanager
def _matmul_precision(allow_tf32: bool):
    """Set torch's float32 matmul precision for the run and restore it (utils.py:57-75)."""
    previous = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("high" if allow_tf32 else "highest")
    with warnings.catch_warnings():
        try:
            yield
        finally:
            torch.set_float32_matmul_precision(previous)


def resolve_sumac_device(S_index: Tensor, S_value: Tensor, config: SumacConfig) -> torch.device:
    """Training device (utils.py:29-46). This implementation runs on CUDA only: a CPU request is
    served by the current CUDA device, and the factors are returned on the requested device."""
    if config.device is not None:
        dev = torch.device(config.device)
    elif S_index.device == S_value.device:
        dev = S_value.device
    elif S_value.device.type != "cpu" and S_index.device.type == "cpu":
        dev = S_value.device
    elif S_index.device.type != "cpu" and S_value.device.type == "cpu":
        dev = S_index.device
    else:
        raise ValueError("S_index and S_value are on different non-CPU devices. "
                         "Pass device=... explicitly to choose the SUMAC training device.")
    return dev


def _cuda_device(requested: torch.device) -> torch.device:
    if requested.type == "cuda":
        return torch.device("cuda", requested.index if requested.index is not None
                            else torch.cuda.current_device())
    if not torch.cuda.is_available():
        raise RuntimeError("sumac_b200 runs on NVIDIA B200 GPUs (sm_100a); no CUDA device is "
                           "available and there is no CPU implementation")
    return torch.device("cuda", torch.cuda.current_device())


def _world_size() -> int:
    import torch.distributed as dist
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def sumac_factorize(*, S_index: Tensor, S_value: Tensor, shape: tuple[int, int],
                    A_init: Tensor | None = None, B_init: Tensor | None = None,
                    config: SumacConfig):
    """Factorize a sparse nonnegative S (COO: S_index (2, nnz), S_value (nnz,)) as ReLU(A B^T).
    Returns (A [m, rank], B [n, rank], history {cost, rmse, jacc, time})."""
    from .gd import GD_loop
    from .salsa import salsa_loop

    S_index_w, S_value_w = S_index, S_value
    if (torch.cuda.is_available() and isinstance(S_index, Tensor) and isinstance(S_value, Tensor)):
        # the data checks (finite, ranges, duplicates: a unique over nnz keys) and the pruning run
        # on the GPU the factorisation will use; the inputs are copied there once
        target = _cuda_device(resolve_sumac_device(S_index, S_value, config))
        S_index_w = S_index.to(target, non_blocking=True)
        S_value_w = S_value.to(target, non_blocking=True)
    m, n = validate_sumac_inputs(S_index=S_index_w, S_value=S_value_w, shape=shape, A_init=A_init,
                                 B_init=B_init, config=config)
    if config.dtype != torch.float32:
        raise NotImplementedError("sumac_b200 computes in float32 (TF32 / 3xTF32 tensor cores); "
                                  "dtype=torch.float64 is not supported")
    with _matmul_precision(config.allow_tf32):
        requested = resolve_sumac_device(S_index, S_value, config)
        S_index, S_value = S_index_w, S_value_w
        # pruning and block sizing are integer work on the input's device, before the GPU is needed
        S_index = S_index.to(S_value.device) if S_index.device != S_value.device else S_index
        S_index, row_mask, col_mask, m_eff, n_eff = prune_zero_rows_cols(S_index, shape=(m, n))
        config.set_block_sizes(m_eff, n_eff)
        dev = _cuda_device(requested)
        config.device = dev
        S_index = S_index.to(dev)
        S_value = S_value.to(device=dev, dtype=config.dtype)
        if row_mask is not None:
            row_mask = row_mask.to(dev)
        if col_mask is not None:
            col_mask = col_mask.to(dev)
        if A_init is not None and B_init is not None:
            A_init = A_init.to(dev)
            B_init = B_init.to(dev)
            if row_mask is not None:
                A_init = A_init[row_mask]
            if col_mask is not None:
                B_init = B_init[col_mask]
        config.print_prefactor_report(S_value, m, n, torch.cuda.device_count())
        if config.method == SumacMethod.GD:
            if _world_size() > 1:
                # one process per GPU: every step's row block split over the process group
                from .shard import sharded_gd_loop
                A, B, costs = sharded_gd_loop(S_index, S_value, m_eff, n_eff, config, A_init,
                                              B_init)
            else:
                A, B, costs = GD_loop(S_index, S_value, m_eff, n_eff, config, A_init, B_init)
        elif config.method == SumacMethod.SALSA:
            if _world_size() > 1:
                # one process per GPU: rows of A and B sharded over the default process group
                from .shard import sharded_salsa_loop
                A, B, costs = sharded_salsa_loop(S_index, S_value, m_eff, n_eff, config, A_init,
                                                 B_init)
            else:
                A, B, costs = salsa_loop(S_index, S_value, m_eff, n_eff, config, A_init, B_init)
        else:
            raise NotImplementedError("method must be chosen from GD or SALSA")
        A_ori, B_ori = restore_zero_rows_cols(A, B, m, n, config.rank, row_mask, col_mask)
        if requested.type != "cuda":
            A_ori, B_ori = A_ori.to(requested), B_ori.to(requested)
        if config.verbose:
            print(f"SUMAC finished after {config.max_iterations} iterations.")
        return A_ori, B_ori, costs
