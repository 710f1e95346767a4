"""CPU oracle for the PagedKV-Fusion hot paths (TEST INFRASTRUCTURE ONLY).

``oracle.oracle`` restates the reference's NumPy algorithms; ``oracle.c_oracle``
loads the C restatement (``pkv_oracle.c``) built by ``oracle/build.py``.
Nothing in the product package imports this directory.
"""

from .oracle import *  # noqa: F401,F403
