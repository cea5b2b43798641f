"""Test configuration: import paths and the ``gpu`` marker.

``ttt-triton_b200/`` (the product, laid out like the reference's top level) and
``oracle/`` (the CPU checker) are put on sys.path. Tests marked ``gpu`` need a CUDA
device and the built library; everything else runs on CPU.
"""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (os.path.join(REPO, "ttt-triton_b200"), os.path.join(REPO, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libttt_b200.so")


def pytest_collection_modifyitems(config, items):
    import pytest
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
