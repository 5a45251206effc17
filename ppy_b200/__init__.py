"""ppy_b200: a B200-native backend for the PPy compiler.

`create_backend` is the `ppy.backends` entry point (`ppy build --backend b200`); it
imports the compiler-side code only when PPy asks for the backend. `runtime.load`
binds what a build wrote and needs no compiler.
"""

from __future__ import annotations

__version__ = "0.1.0"

__all__ = ["__version__", "create_backend"]


def create_backend(options=None):
    """The `b200` backend, given its `[tool.ppy.backends.b200]` table."""
    from .backend import B200Backend

    return B200Backend(options)
