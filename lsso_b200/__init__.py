"""B200 (sm_100a) implementation of the LSSO token mixer.

Drop-in for the public API of Yang916-yy/LSSO (``lsso/__init__.py``):
``LSSO``, ``LSSOConfig``, ``CoreMode`` and ``__version__``; the same objects
are importable as ``lsso``.
"""

from .ball import CoreMode, LSSO, LSSOConfig

__version__ = "0.6.3"

__all__ = ["CoreMode", "LSSO", "LSSOConfig", "__version__"]
