"""``mace_ictc.hp.runtime`` (reference ``mace_ictc/hp/runtime.py:7,84,123,132``): the
same four functions, implemented in ``mace_ictc.runtime``."""
from mace_ictc.runtime import check_model, configure_model, create_model, energy_and_forces

__all__ = ["create_model", "energy_and_forces", "check_model", "configure_model"]
