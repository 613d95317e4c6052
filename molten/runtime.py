"""Import-compatible alias of ``molten.runtime``: the implementation is ``molten_b200.runtime``."""
from molten_b200.runtime import *  # noqa: F401,F403
