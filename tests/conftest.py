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


_RECORDS = []


def rel_err(a, ref):
    """max|a - ref| / max|ref| (the parity metric). With M3_PARITY_LOG set, every value is
    also recorded (test id, calling line, the caller's loop key ``k`` if any) and written
    as JSON lines to that file at the end of the session: the achieved-error record."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref)) if ref.size else 0.0
    err = float(np.max(np.abs(a - ref)) / (den if den > 0 else 1.0)) if ref.size else 0.0
    if os.environ.get("M3_PARITY_LOG"):
        import inspect
        fr = inspect.currentframe().f_back
        key = fr.f_locals.get("k") if fr is not None else None
        _RECORDS.append({"test": os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0],
                         "line": fr.f_lineno if fr is not None else None,
                         "key": key if isinstance(key, str) else None, "err": err})
    return err


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("M3_PARITY_LOG")
    if path and _RECORDS:
        import json
        with open(path, "a") as f:
            for r in _RECORDS:
                f.write(json.dumps(r) + "\n")


@pytest.fixture(scope="session")
def golden():
    return load_golden
