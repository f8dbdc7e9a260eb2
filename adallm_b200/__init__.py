"""adallm_b200: B200-native (sm_100a) kernels for the decode hot path of the
AdaLLM NVFP4 inference runtime -- the NVFP4 linear op and FP8 paged decode
attention, with the FP8 KV-cache store, rotary embedding, RMSNorm and gated
activations beside them -- behind a C ABI (include/adallm_b200.h) and a thin
Python layer that mirrors the reference's ``adallm.ops`` interfaces.

Build the CUDA library with ``python -m adallm_b200.build``.  No CPU or
PyTorch fallback exists: ops raise if the library is missing.
"""
from . import _native  # noqa: F401
from .install import install  # noqa: F401

__all__ = ["_native", "install"]
