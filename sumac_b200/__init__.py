"""sumac_b200 — B200 (sm_100a) implementation of sumac's hot path (fused masked ReLU product,
SALSA and GD block steps) behind sumac's public API:

    from sumac_b200 import sumac_factorize, SumacConfig, SumacMethod
"""
from .config import AutotuneMode, OptimizerName, SumacConfig, SumacMethod
from .sumac import sumac_factorize

__all__ = ["sumac_factorize", "SumacConfig", "SumacMethod", "OptimizerName", "AutotuneMode"]
