"""Loader of the two in-tree native extensions.

``_C`` holds the sm_100a kernels and the symmetric-memory layer, ``_cpu`` the
host runtime (CPU mailbox engine, FD exchange). Both are built in place by
``python setup.py build_ext --inplace``. On a machine with a GPU a missing
``_C`` is an error (there is no silent PyTorch fallback for the kernels).
"""
import importlib

_C = None
_cpu = None


class NativeExtensionMissing(ImportError):
    pass


def _pkg():
    return __name__.rsplit(".", 1)[0]


def cuda_ext():
    """Return the CUDA extension module, raising if it was not built."""
    global _C
    if _C is None:
        import torch  # noqa: F401 - loads libc10 / libtorch, which the extension links against

        try:
            _C = importlib.import_module(f"{_pkg()}._C")
        except ImportError as e:  # pragma: no cover - depends on the build
            raise NativeExtensionMissing(
                "the sm_100a extension (_C) is not built: run `python setup.py build_ext --inplace` "
                f"in the repository root ({e})"
            ) from e
    return _C


def cpu_ext():
    """Return the host-runtime extension module, raising if it was not built."""
    global _cpu
    if _cpu is None:
        import torch  # noqa: F401 - as above

        try:
            _cpu = importlib.import_module(f"{_pkg()}._cpu")
        except ImportError as e:  # pragma: no cover
            raise NativeExtensionMissing(
                "the host runtime extension (_cpu) is not built: run `python setup.py build_ext --inplace` "
                f"({e})"
            ) from e
    return _cpu
