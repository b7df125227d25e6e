"""Adaptive Precision Ascension on B200.

Drop-in for the reference package ``apa``: the same public names
(apa/__init__.py:1-15), with APALinear's casts, GEMMs and telemetry and the
manager's ladder running as sm_100a kernels from libapa_kernels.so.
"""
from .config import APAConfig
from .layers import APALinear, APABoundaryCast
from .manager import APAManager
from .telemetry import APAForensicLogger

__version__ = "0.1.0"

__all__ = [
    "APAConfig",
    "APALinear",
    "APABoundaryCast",
    "APAManager",
    "APAForensicLogger",
    "__version__",
]
