"""openquant.cli -> openquant_b200.cli (reference module path)."""
from openquant_b200.cli import *  # noqa: F401,F403
from openquant_b200.cli import __all__  # noqa: F401
