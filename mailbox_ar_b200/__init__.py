"""Importable name of the ``3080_mod_p2p_sglang_patch_b200`` package.

That package's name starts with a digit, so ``import`` statements cannot
spell it. Here ``import mailbox_ar_b200.engine`` or ``from
mailbox_ar_b200.engine import LLMEngine`` resolve to the same module objects
as ``importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine")``, not
copies: one set of extension modules, one set of per-process state.
"""
import importlib
import importlib.abc
import importlib.util
import sys

_REAL = "3080_mod_p2p_sglang_patch_b200"
_ALIAS = __name__


class _AliasFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """``mailbox_ar_b200.X`` -> the already imported ``3080_...X``."""

    def find_spec(self, name, path, target=None):
        if name.startswith(_ALIAS + "."):
            return importlib.util.spec_from_loader(name, self)
        return None

    def create_module(self, spec):
        return importlib.import_module(_REAL + spec.name[len(_ALIAS):])

    def exec_module(self, module):
        pass  # the real module is already executed


if not any(isinstance(f, _AliasFinder) for f in sys.meta_path):
    sys.meta_path.insert(0, _AliasFinder())

_pkg = importlib.import_module(_REAL)
globals().update({k: v for k, v in vars(_pkg).items() if not k.startswith("__")})
