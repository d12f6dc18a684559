"""openquant.groupwise -> openquant_b200.groupwise (reference module path)."""
from openquant_b200.groupwise import *  # noqa: F401,F403
from openquant_b200.groupwise import __all__  # noqa: F401
