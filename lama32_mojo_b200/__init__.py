"""lama32_mojo_b200 — B200-native (sm_100a) INT8 group-quantized (W8A32, group 64)
decode/prefill path, a drop-in for plutonium-guy/lama32_mojo's Q8 path.

Compute lives in ``libq8cuda.so`` (C ABI in ``include/q8cuda.h``); this package
is the host side: ``model.Q8Model`` (the reference's model-shell API),
``ops`` (op-level kernels on CUDA tensors) and ``config`` (model dimensions).
"""
from .config import Config, PRESETS  # noqa: F401

__all__ = ["Config", "PRESETS"]
