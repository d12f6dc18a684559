"""openquant.group_benchmark -> openquant_b200.group_benchmark (reference module path)."""
from openquant_b200.group_benchmark import *  # noqa: F401,F403
from openquant_b200.group_benchmark import __all__  # noqa: F401
