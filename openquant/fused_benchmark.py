"""openquant.fused_benchmark -> openquant_b200.fused_benchmark (reference module path)."""
from openquant_b200.fused_benchmark import *  # noqa: F401,F403
from openquant_b200.fused_benchmark import __all__  # noqa: F401
