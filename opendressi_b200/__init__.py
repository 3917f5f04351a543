"""opendressi_b200 -- the Dressi-AD per-iteration hot path on NVIDIA B200.

Layers (bottom up):
  csrc/ + libdressi_b200.so  hand-written sm_100a kernels behind a C ABI
                             (include/dressi_b200.h)
  _native                    ctypes binding of that ABI (no fallback)
  ops                        op-level calls on torch CUDA tensors
  plans                      fused fwd+bwd+Adam iterations as CUDA graphs
  scene                      seeded synthetic workloads (configs C1-C5)
"""

from ._native import DressiError, load as load_library  # noqa: F401
from . import scene  # noqa: F401

__all__ = ["DressiError", "load_library", "scene", "ops", "plans"]


def __getattr__(name):
    # ops / plans import torch; load them on first use
    if name in ("ops", "plans"):
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
