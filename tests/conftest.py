import atexit
import os
import pathlib
import shutil
import sys
import tempfile

import numpy as np
import pytest

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
for p in (str(HERE), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

# Specialised tile kernels compiled during the tests go to a cache of the
# session's own (set before the library is loaded), not the user's.
if "SIMTGO_B200_CACHE" not in os.environ:
    _cache = tempfile.mkdtemp(prefix="simtgo_b200_cache_")
    os.environ["SIMTGO_B200_CACHE"] = _cache
    atexit.register(shutil.rmtree, _cache, True)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    with np.load(HERE / "golden" / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden
