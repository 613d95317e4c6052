"""Import-compatible alias of ``molten.codegen``: the implementation is ``molten_b200.codegen``."""
from molten_b200.codegen import *  # noqa: F401,F403
