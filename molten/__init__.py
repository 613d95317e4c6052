"""Import-compatible alias package: ``import molten`` resolves to molten_b200.

Lets code written against the reference (``from molten.ir import
DataflowGraph``, ``from molten.codegen import compile_graph`` ...) run
unchanged on the sm_100a backend.
"""
from molten_b200 import *  # noqa: F401,F403
from molten_b200 import __version__  # noqa: F401
