"""unsloth_spectral -- B200-native (sm_100a) compressed-KV decode path.

Drop-in for the reference package's decode path: same public names
(unsloth_spectral/__init__.py:76-108 of the reference), backed by ``libspx.so``:
``SpectralCache``, ``SpectralBlock``, ``spectral_attention_forward``,
``validate_spectral_attention``, ``patch_unsloth_attention``, ``get_cache_stats``,
``TRITON_AVAILABLE`` / ``TRITON_VERSION`` and, when the library loads,
``spectral_attention_decode`` and ``TritonSpectralConfig``.
Set ``UNSLOTH_SPECTRAL_QUIET=1`` to silence the import banner.
"""
import os

__version__ = "0.1.0+b200"

from .spectral_cache import SpectralBlock, SpectralCache  # noqa: E402
from .spectral_attention import spectral_attention_forward, validate_spectral_attention  # noqa: E402
from .integration import get_cache_stats, patch_unsloth_attention  # noqa: E402
from .kernels import TRITON_AVAILABLE, TRITON_VERSION  # noqa: E402
from .rsvd import batched_randomized_svd  # noqa: E402

__all__ = [
    "SpectralCache",
    "SpectralBlock",
    "spectral_attention_forward",
    "validate_spectral_attention",
    "patch_unsloth_attention",
    "get_cache_stats",
    "batched_randomized_svd",
    "TRITON_AVAILABLE",
    "TRITON_VERSION",
]

if TRITON_AVAILABLE:
    from .kernels import TritonSpectralConfig, spectral_attention_decode  # noqa: E402,F401
    __all__.extend(["spectral_attention_decode", "TritonSpectralConfig"])


def print_banner():
    print("=" * 70)
    print(f"  UNSLOTH SPECTRAL v{__version__}  (sm_100a CUDA: {'loaded' if TRITON_AVAILABLE else 'MISSING'})")
    print("=" * 70)


if not os.environ.get("UNSLOTH_SPECTRAL_QUIET"):
    print_banner()
