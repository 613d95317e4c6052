"""Import-compatible alias of ``molten.compiler``: the implementation is ``molten_b200.compiler``."""
from molten_b200.compiler import *  # noqa: F401,F403
