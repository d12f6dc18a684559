"""openquant.autotune -> openquant_b200.autotune (reference module path)."""
from openquant_b200.autotune import *  # noqa: F401,F403
from openquant_b200.autotune import __all__  # noqa: F401
