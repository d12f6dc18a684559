"""openquant.benchmark -> openquant_b200.benchmark (reference module path)."""
from openquant_b200.benchmark import *  # noqa: F401,F403
from openquant_b200.benchmark import __all__  # noqa: F401
