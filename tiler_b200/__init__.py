"""tiler_b200 — B200-native (sm_100a) execution backend for moderately-ai/tiler's
registered operation families, behind a C-ABI (include/tiler_cuda.h).

Layers:
  * ``libtiler_cuda.so`` (tiler_b200/csrc): the kernels and the C-ABI;
  * :mod:`tiler_b200.families`: torch-facing entry points per family;
  * :mod:`tiler_b200.adapter`: the RuntimeAdapter phases over the C-ABI;
  * :mod:`tiler_b200.provider`: the reduction groupings the backend declares;
  * :mod:`tiler_b200.sharding`: one-process-per-GPU row / N sharding.
"""
from . import _native  # noqa: F401

__all__ = ["families", "adapter", "provider", "sharding"]
