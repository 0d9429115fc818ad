#!/usr/bin/env python3
"""Training / evaluation entry point (``nano_qwen_b200.cli``)."""

import sys

from nano_qwen_b200.cli import main

if __name__ == "__main__":
    sys.exit(main())
