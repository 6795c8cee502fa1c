"""Import name ``hs_guard_b200`` for the package whose sources live in ``hs-guard_b200/``.

A hyphen cannot appear in a Python module name, so this module turns itself into a package rooted at
that directory: ``import hs_guard_b200.runtime`` loads ``hs-guard_b200/runtime.py``.
"""
import os as _os

__path__ = [_os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "hs-guard_b200")]

from hs_guard_b200.config import DEFAULT, HsgConfig, LABELS, ROLES  # noqa: E402,F401


def __getattr__(name):
    # StreamingGuard pulls in torch and the CUDA library; resolve it lazily.
    if name == "StreamingGuard":
        from hs_guard_b200.runtime import StreamingGuard
        return StreamingGuard
    raise AttributeError(name)
