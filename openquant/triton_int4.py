"""openquant.triton_int4 -> openquant_b200.triton_int4 (reference module path)."""
from openquant_b200.triton_int4 import *  # noqa: F401,F403
from openquant_b200.triton_int4 import __all__  # noqa: F401
