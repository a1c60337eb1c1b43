"""B200 (sm_100a) implementation of the FastWAM per-action-chunk denoising path.

Import with ``importlib.import_module("faster-action-models_b200")`` after
putting the repository root on ``sys.path`` (the directory name is not a
Python identifier).
"""
from ._lib import FamError, lib, version  # noqa: F401
