"""sumac_b200 — B200 (sm_100a) implementation of sumac's hot path (fused masked ReLU product,
SALSA and GD block steps) behind sumac's public API."""
from . import ops  # noqa: F401
