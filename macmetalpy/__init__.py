"""``import macmetalpy`` answers with the B200 backend (``macmetalpy_b200``).

The reference is imported as ``import macmetalpy as cp`` (its tests and its
users do, e.g. ``tests/test_fusion.py:6``).  This package makes that name a
drop-in for the hot path: ``macmetalpy`` *is* the ``macmetalpy_b200``
module, and every submodule ``macmetalpy.X`` is the module object
``macmetalpy_b200.X`` (one copy: ``macmetalpy._config.get_config()`` returns
the same singleton as ``macmetalpy_b200._config.get_config()``).
"""

from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys

import macmetalpy_b200 as _impl

_ALIAS, _REAL = "macmetalpy", "macmetalpy_b200"


class _SubmoduleAlias(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """Resolves ``macmetalpy.X`` to the already-importable ``macmetalpy_b200.X``."""

    def find_spec(self, fullname, path=None, target=None):
        if not fullname.startswith(_ALIAS + "."):
            return None
        real = _REAL + fullname[len(_ALIAS):]
        if importlib.util.find_spec(real) is None:
            return None
        return importlib.util.spec_from_loader(fullname, self)

    def create_module(self, spec):
        return importlib.import_module(_REAL + spec.name[len(_ALIAS):])

    def exec_module(self, module):
        pass  # the real module has already run


if not any(isinstance(f, _SubmoduleAlias) for f in sys.meta_path):
    sys.meta_path.insert(0, _SubmoduleAlias())
sys.modules[__name__] = _impl
