"""Drop-in solution file: the same module name and entry point as the reference
(``kernel.py::run`` of nikhilnd/mlsys26-flashinfer-moe), backed by the sm_100a
kernels of ``moe_b200``.  A harness that imports the reference's ``kernel.py``
and calls ``run(...)`` can import this file instead.
"""
import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

from moe_b200.api import run  # noqa: E402,F401

__all__ = ["run"]
