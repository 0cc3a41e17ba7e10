"""Shared pytest setup: the ``gpu`` marker and import paths.

The package directory ``rust-llm-pager_b200/`` is not an importable Python
name, so its contents (the ``pager_hf`` drop-in package) are put on
``sys.path`` here, as are the repository root (for ``oracle``) and
``tests/golden`` (for the seeded case builders).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "rust-llm-pager_b200"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
