"""Loader for the in-tree sm_100a extension ``nano_qwen_b200._C``.

CUDA tensors always go to the native kernels; there is no silent fallback.
If the extension is missing on a machine with a GPU, the first CUDA op
raises with the build command.
"""

from __future__ import annotations

_EXT = None
_ERR = None


def ext():
    global _EXT, _ERR
    if _EXT is None:
        try:
            from nano_qwen_b200 import _C  # noqa: F401
            _EXT = _C
        except ImportError as e:  # pragma: no cover - depends on build state
            _ERR = e
            raise RuntimeError(
                "nano_qwen_b200._C (sm_100a kernels) is not built or failed to load: "
                f"{e}.  Build it with `python setup.py build_ext --inplace`."
            ) from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
