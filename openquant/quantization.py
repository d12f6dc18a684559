"""openquant.quantization -> openquant_b200.quantization (reference module path)."""
from openquant_b200.quantization import *  # noqa: F401,F403
from openquant_b200.quantization import __all__  # noqa: F401
