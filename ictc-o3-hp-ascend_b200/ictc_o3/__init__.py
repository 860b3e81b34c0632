"""ICTC-O3 operators on a B200-native (sm_100a) CUDA backend.

The package exports the public operators as the reference's does
(``ictc_o3/__init__.py``: ``from ictc_o3 import EdgeTensorProduct``, ...).  The
reference's mesh electrostatics are not part of this backend.
"""
from .operators import *  # noqa: F401,F403
from .operators import __all__

__version__ = "0.1.0"
