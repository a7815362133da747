import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "mamba3-ssm_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    """Load tests/golden/<name>.npz. uint16 arrays hold raw bf16 bit patterns and are
    returned as float64 numpy arrays of the bf16 values; ``bf16`` lists those keys."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    out, bf = {}, set()
    for k in z.files:
        a = z[k]
        if a.dtype == np.uint16:
            a = (a.astype(np.uint32) << 16).view(np.float32)
            bf.add(k)
        out[k] = a
    out["bf16"] = bf
    return out


def rel_err(a, ref):
    """max|a - ref| / max|ref| (the parity metric)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(a - ref)) / (den if den > 0 else 1.0))


@pytest.fixture(scope="session")
def golden():
    return load_golden
