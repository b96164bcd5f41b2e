"""Configuration object with the reference's fields, defaults and validation
(src/sumac/config/options.py:14-296), plus opt-in fields for this implementation."""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, fields
from enum import Enum
from pathlib import Path

import torch


def _validate_finite_number(name: str, value) -> None:
    if not math.isfinite(value):
        raise ValueError(f"{name} must be a finite number, got {value!r}")


class SumacMethod(Enum):
    """SALSA (stochastic alternating least squares) or GD (gradient descent)."""
    SALSA = "salsa"
    GD = "gd"


class OptimizerName(Enum):
    ADAM = "adam"
    ADAMW = "adamw"
    SGD = "sgd"
    MUON = "muon"


class AutotuneMode(Enum):
    """Accepted for API compatibility. This implementation has no autotuner: every kernel uses a
    fixed configuration per rank, so the mode is ignored."""
    CACHE = "cache"
    FORCE = "force"
    DISABLE = "disable"
    FALLBACK = "fallback"


def default_kernel_autotune_cache_dir() -> Path:
    xdg_cache_home = os.environ.get("XDG_CACHE_HOME")
    if xdg_cache_home:
        return Path(xdg_cache_home) / "sumac"
    return Path.home() / ".cache" / "sumac"


@dataclass(kw_only=True)
class SumacConfig:
    """Same fields and defaults as sumac's SumacConfig (options.py:45-157).

    Additional opt-in fields (defaults keep the reference's behaviour):
      perm_device: device of the random generators, the ones that draw the row permutations and
        the one that draws the initial factors (default: the training device, as the reference).
        "cpu" reproduces the random draws of a CPU run of the reference; the arithmetic still runs
        on the training device.
      tf32_mode: None (follow allow_tf32: TF32 if True, 3xTF32 fp32-accurate otherwise), or one of
        "tf32", "3xtf32".
      keep_best: SALSA returns the evaluated iterate of lowest cost, refactored (the MATLAB
        implementation's finish, matlab/sumac/salsa_loop.m:61-79), instead of the last iterate.
      report_fnnz: SALSA adds "fnnz" to the history: the fraction nnz(ReLU(A B^T)) / nnz(S) that
        the MATLAB implementation reports (matlab/sumac/compute_errors.m:62).
    """
    method: SumacMethod = SumacMethod.SALSA
    rank: int = 16
    max_iterations: int = 25
    num_blocks: int | None = None
    cols_per_block: int | None = None
    seed: int | None = None
    cache_mb: int = 5000
    dtype: torch.dtype = torch.float32
    allow_tf32: bool = False
    device: torch.device | None = None
    momentum: float = -1.0
    learning_rate: float = 1e-1
    verbose: bool = True
    eval_interval: int | None = None
    optimizer: OptimizerName = OptimizerName.ADAM
    adam_betas: tuple[float, float] = (0.9, 0.999)
    adam_eps: float = 1e-8
    shuffle_blocks: bool = False
    batch_blocks: int = 1
    autotune: AutotuneMode = AutotuneMode.CACHE
    autotune_cache_dir: str | Path | None = None
    autotune_verbose: bool = False
    input_filename: str | None = None
    log_filename: str | None = None
    # opt-in extensions
    perm_device: str | torch.device | None = None
    tf32_mode: str | None = None
    keep_best: bool = False
    report_fnnz: bool = False

    def __post_init__(self):
        self._validate_integer_options()
        self._validate_numeric_options()
        if self.eval_interval is None:
            self.eval_interval = 100 if self.method == SumacMethod.GD else 10
        if self.eval_interval <= 0:
            raise ValueError(
                f"eval_interval must be a positive integer or None, got {self.eval_interval!r}")
        if self.autotune_cache_dir is None:
            self.autotune_cache_dir = default_kernel_autotune_cache_dir()
        self.autotune_cache_dir = str(self.autotune_cache_dir)
        if self.momentum < 0:
            self.momentum = 0.7
            if self.optimizer == OptimizerName.MUON and self.method == SumacMethod.GD:
                self.momentum = 0.95
        if not 0 <= self.momentum < 1:
            raise ValueError(f"momentum must satisfy 0 <= momentum < 1, got {self.momentum!r}")
        self._validate_adam_options()
        if self.tf32_mode not in (None, "tf32", "3xtf32"):
            raise ValueError(f"tf32_mode must be None, 'tf32' or '3xtf32', got {self.tf32_mode!r}")
        if self.seed is not None and self.verbose:
            print(f"seed = {self.seed}")

    def _validate_integer_options(self) -> None:
        if self.rank <= 0:
            raise ValueError(f"rank must be a positive integer, got {self.rank!r}")
        if self.max_iterations < 0:
            raise ValueError(
                f"max_iterations must be a nonnegative integer, got {self.max_iterations!r}")
        if self.num_blocks is not None and self.num_blocks < 1:
            raise ValueError(f"num_blocks must be a positive integer or None, got {self.num_blocks!r}")
        if self.batch_blocks <= 0:
            raise ValueError(f"batch_blocks must be a positive integer, got {self.batch_blocks!r}")

    def _validate_numeric_options(self) -> None:
        _validate_finite_number("cache_mb", self.cache_mb)
        if self.cache_mb <= 0:
            raise ValueError(f"cache_mb must be positive, got {self.cache_mb!r}")
        if self.dtype not in (torch.float32, torch.float64):
            raise TypeError(f"dtype must be torch.float32 or torch.float64, got {self.dtype!r}")
        if self.dtype == torch.float64 and self.allow_tf32:
            raise ValueError("dtype=torch.float64 and allow_tf32=True are mutually exclusive")
        _validate_finite_number("learning_rate", self.learning_rate)
        if self.learning_rate < 0:
            raise ValueError(f"learning_rate must be nonnegative, got {self.learning_rate!r}")
        _validate_finite_number("momentum", self.momentum)

    def _validate_adam_options(self) -> None:
        if self.method != SumacMethod.GD or self.optimizer not in (OptimizerName.ADAM,
                                                                   OptimizerName.ADAMW):
            return
        _validate_finite_number("adam_eps", self.adam_eps)
        if self.adam_eps <= 0:
            raise ValueError(f"adam_eps must be positive, got {self.adam_eps!r}")
        for beta in self.adam_betas:
            _validate_finite_number("adam_betas value", beta)
            if not 0 <= beta < 1:
                raise ValueError(f"adam_betas values must satisfy 0 <= beta < 1, got {self.adam_betas!r}")

    def set_block_sizes(self, m: int, n: int):
        """Block count from the cache budget when unset (options.py:253-267)."""
        if self.num_blocks is None:
            max_bytes = self.cache_mb * 1e6
            bytes_per_dtype = 8 if self.dtype == torch.float64 else 4
            self.cols_per_block = max(1, int(max_bytes // (m * bytes_per_dtype)))
            self.num_blocks = math.ceil(n / self.cols_per_block)
        max_num_blocks = min(m, n)
        if self.num_blocks > max_num_blocks:
            raise ValueError(
                "num_blocks must satisfy "
                f"1 <= num_blocks <= min(effective shape)={max_num_blocks}, got {self.num_blocks}")
        self.cols_per_block = int(n // self.num_blocks)

    def print_prefactor_report(self, S_value, m: int, n: int, devcount: int):
        if not self.verbose:
            return
        print(f"\n  Input to SUMAC is a {m}x{n} sparse matrix with {len(S_value)} nonzeros.")
        print(f"  Attempting matrix completion with rank {self.rank}.")
        print(f"  Available GPUs: {devcount}.")
        print("  Options:")
        print("\n".join(f"    {f.name}: {getattr(self, f.name)}" for f in fields(self)))
        print()

    def get_generator(self):
        """(gen, gen_rows, gen_aux) seeded seed, seed+1, seed+2 (options.py:282-296). The first
        two live on the training device; the third on it for SALSA and on the CPU for GD.
        With perm_device set, the generators live there instead."""
        dev = self.perm_device if self.perm_device is not None else self.device
        gen = torch.Generator(device=dev)
        gen_rows = torch.Generator(device=dev)
        tmp_device = dev if self.method == SumacMethod.SALSA else "cpu"
        gen_aux = torch.Generator(device=tmp_device)
        generators = (gen, gen_rows, gen_aux)
        if self.seed is None:
            for g in generators:
                g.seed()
        else:
            for offset, g in enumerate(generators):
                g.manual_seed(self.seed + offset)
        return generators

    def precision(self) -> int:
        from ._native import SUMAC_3XTF32, SUMAC_TF32
        if self.tf32_mode == "tf32":
            return SUMAC_TF32
        if self.tf32_mode == "3xtf32":
            return SUMAC_3XTF32
        return SUMAC_TF32 if self.allow_tf32 else SUMAC_3XTF32
