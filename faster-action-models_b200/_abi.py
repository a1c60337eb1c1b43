"""ctypes declarations of the model-level entry points of include/fam.h."""
from __future__ import annotations

import ctypes as C


def declare(lib) -> None:
    return None
