"""Loads the reference's compiled OpenMP prefix-mean kernel from oracle/_ref.

TEST INFRASTRUCTURE / CPU BASELINE ONLY.  ``oracle/Makefile`` builds
``oracle/_ref/race_pref*.so`` from ``kernels/cpu/race_pref.cpp`` of the
reference; the module exposes ``race_prefix_mean_flat`` and
``race_prefix_mean_flat_bw`` (race_pref.cpp:222-226).
"""
import os
import sys

_REF = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def load_race_pref():
    """Return the compiled reference module, or None when it was not built."""
    import glob
    if not glob.glob(os.path.join(_REF, "race_pref*.so")):
        return None
    import torch  # noqa: F401  (libtorch must be loaded first)
    if _REF not in sys.path:
        sys.path.insert(0, _REF)
    try:
        import race_pref
    except ImportError:
        return None
    return race_pref
