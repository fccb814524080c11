"""ferrite-strata_b200: a B200 (sm_100a) execution backend for Ferrite Strata.

The product is ``libstrata_b200.so`` (built from ``csrc/`` by ``build.py``),
which exports the reference's plugin ABI symbol ``strata_plugin_v1``.  The
``strata_host`` package drives it from Python the way the reference's Rust
host does.
"""
import os as _os
import sys as _sys

HERE = _os.path.dirname(_os.path.abspath(__file__))
LIBRARY = _os.path.join(HERE, "libstrata_b200.so")
if HERE not in _sys.path:
    _sys.path.insert(0, HERE)
