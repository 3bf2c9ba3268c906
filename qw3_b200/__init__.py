"""qw3_b200 — B200 (sm_100a) backend for the qw3 engine's fused per-layer path.

The product is the C-ABI library ``libds3cuda.so`` (declared in
include/ds3_cuda.h). This package holds its CUDA sources (``csrc/``), the
nvcc build (``build.py``), the Python mirror of the C-ABI (``ds3.py``), the
shared synthetic-input generators (``inputs.py``) and the row-shard planner
for multi-GPU runs (``shard.py``).
"""

from . import ds3  # noqa: F401

__all__ = ["ds3"]
