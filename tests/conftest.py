"""Shared test setup.

* Marker `gpu`: the test needs a CUDA device (run with `-m gpu` on a B200; `-m "not gpu"` runs the
  CPU suite).  Without a CUDA device a gpu-marked test is skipped, never silently passed.
* The repository root is importable (modelcore_b200, oracle).  modelcore itself -- the reference
  whose API the decode path plugs into -- is imported from the environment if installed, else
  from the repository's baseline/_ref install of it.
"""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)
_REF = os.path.join(REPO, "baseline", "_ref")
try:
    import modelcore  # noqa: F401
except ImportError:
    if os.path.isdir(_REF):
        sys.path.append(_REF)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); deselect with -m 'not gpu'")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def golden_files(prefix):
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))


def have_modelcore():
    try:
        import modelcore  # noqa: F401
        return True
    except ImportError:
        return False
