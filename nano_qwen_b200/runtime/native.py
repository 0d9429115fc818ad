"""Host-side native runtime (C++, ``nano_qwen_b200._runtime``).

``TokenWindowReader(files, itemsize, pad=0)``: memory-mapped token shards
served as int64 windows of their concatenation, gathered in C++ with the GIL
released (csrc/runtime/token_reader.cpp).
"""

from __future__ import annotations

from .. import _runtime  # noqa: F401  (ImportError when the extension is not built)

TokenWindowReader = _runtime.TokenWindowReader
