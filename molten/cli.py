"""Import-compatible alias of ``molten.cli``: the implementation is ``molten_b200.cli``
(``python -m molten.cli compile graph.json -o out/``)."""
import sys

from molten_b200.cli import *  # noqa: F401,F403
from molten_b200.cli import main

if __name__ == "__main__":
    sys.exit(main() or 0)
