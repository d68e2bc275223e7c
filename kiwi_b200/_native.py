"""Loader for the in-tree native extension ``kiwi_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).  Import fails loudly when it is missing: there is
no pure-Python fallback for any GPU path.
"""
import importlib

_C = None


def load():
    """The extension module kiwi_b200._C (imported once; ImportError if not built)."""
    global _C
    if _C is None:
        import torch  # noqa: F401  (loads libc10/libtorch the extension links against)

        try:
            _C = importlib.import_module("kiwi_b200._C")
        except ImportError as e:  # pragma: no cover - exercised only on a broken build
            raise ImportError(
                "kiwi_b200 native extension is not built; run `python setup.py build_ext --inplace` "
                f"at the repository root ({e})"
            ) from e
    return _C
