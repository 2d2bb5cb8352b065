"""Decode kernels for the spectral cache (sm_100a CUDA through ``libspx.so``).

Keeps the reference module's names (unsloth_spectral/kernels/__init__.py:38-67):
``TRITON_AVAILABLE`` is true whenever the CUDA library loads, so callers that route on
it (integration.py:33-36, :636) take this path; ``TRITON_VERSION`` reports the
library's ABI version.
"""
import logging

from .. import _native

logger = logging.getLogger("unsloth_spectral.kernels")

TRITON_AVAILABLE = _native.available()
TRITON_VERSION = f"spx-sm100a-abi{_native.ABI_VERSION}" if TRITON_AVAILABLE else None

from .spectral_attention import (  # noqa: E402
    TritonSpectralConfig,
    spectral_attention_decode,
    spectral_attention_decode_pytorch,
    spectral_score_forward,
    spectral_value_forward,
)

__all__ = [
    "spectral_attention_decode",
    "spectral_score_forward",
    "spectral_value_forward",
    "TritonSpectralConfig",
    "TRITON_AVAILABLE",
    "TRITON_VERSION",
]
