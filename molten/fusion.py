"""Import-compatible alias of ``molten.fusion``: the implementation is ``molten_b200.fusion``."""
from molten_b200.fusion import *  # noqa: F401,F403
