"""Python access to the C++ serving runtime (extension ``_sp_core``).

``core()`` returns the compiled module; ``StatusError`` is the exception type
its entry points raise (``.code`` = numeric status, ``.status`` = its name).
"""
from __future__ import annotations

from .. import _ext


def core():
    return _ext.core()


def __getattr__(name):
    if name == "StatusError":
        return core().StatusError
    raise AttributeError(name)
