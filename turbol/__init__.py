"""``import turbol``: the reference's package name for this framework.

The reference's users write ``import turbol`` (turbol_vllm/python/setup.cfg:6,
turbol_vllm/python/turbol/__init__.py:10-211).  This package makes that name
resolve to :mod:`turbol_b200`: ``turbol`` *is* the ``turbol_b200`` module object,
and ``turbol.<sub>`` (``turbol.turbol_core``, ``turbol.vllm_inference``,
``turbol.rl.ppo`` ...) is the same module object as ``turbol_b200.<sub>``, so
the native extension is loaded once and its types are shared.

The framework's own code imports ``turbol_b200``; a process that puts another
``turbol`` package first on ``sys.path`` (the reference build used as a
baseline) gets that one instead, and nothing here runs.
"""
from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys

_IMPL = "turbol_b200"
_impl = importlib.import_module(_IMPL)


class _AliasLoader(importlib.abc.Loader):
    def __init__(self, target: str):
        self.target = target

    def create_module(self, spec):
        return importlib.import_module(self.target)

    def exec_module(self, module):  # the target module is already executed
        pass


class _AliasFinder(importlib.abc.MetaPathFinder):
    """Resolves ``turbol.<sub>`` to the already importable ``turbol_b200.<sub>``."""

    def find_spec(self, fullname, path=None, target=None):
        if not fullname.startswith(__name__ + "."):
            return None
        real = _IMPL + fullname[len(__name__):]
        if importlib.util.find_spec(real) is None:
            return None
        return importlib.util.spec_from_loader(fullname, _AliasLoader(real))


if not any(isinstance(f, _AliasFinder) for f in sys.meta_path):
    sys.meta_path.insert(0, _AliasFinder())
for _name, _mod in list(sys.modules.items()):
    if _name.startswith(_IMPL + "."):
        sys.modules.setdefault(__name__ + _name[len(_IMPL):], _mod)
sys.modules[__name__] = _impl
