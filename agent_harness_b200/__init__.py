"""agent_harness_b200 — B200 (sm_100a) implementation of agent_harness's
quantized-weight hot path behind a C ABI (include/ah_cuda.h).

  kernels  : device-tensor front-end (dequant, conversion, quantisers, fused GEMV)
  hostapi  : host-slice mirrors of the reference's Rust functions
"""
from ._lib import AhError, LIB_PATH, lib  # noqa: F401

__all__ = ["AhError", "LIB_PATH", "lib"]
