"""CPU checkers for the k-quant dequantize-and-multiply path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this package.  The product (``vibeblade_b200``) never does.
"""
from .oracle import Oracle, RefLib, load_oracle, load_ref  # noqa: F401
