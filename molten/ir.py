"""Import-compatible alias of ``molten.ir``: the implementation is ``molten_b200.ir``."""
from molten_b200.ir import *  # noqa: F401,F403
