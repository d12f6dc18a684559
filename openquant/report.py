"""openquant.report -> openquant_b200.report (reference module path)."""
from openquant_b200.report import *  # noqa: F401,F403
from openquant_b200.report import __all__  # noqa: F401
