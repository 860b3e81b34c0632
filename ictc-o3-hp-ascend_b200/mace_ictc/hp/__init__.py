"""The reference's model API import path (``mace_ictc/hp/__init__.py``): the public
ICTC-O3 operators and the model runtime (``create_model``, ``configure_model``,
``check_model``, ``energy_and_forces`` from ``mace_ictc.runtime``)."""
from ictc_o3 import *  # noqa: F401,F403
from ictc_o3 import __all__ as _operators

from .runtime import check_model, configure_model, create_model, energy_and_forces

__all__ = [*_operators, "check_model", "configure_model", "create_model", "energy_and_forces"]
