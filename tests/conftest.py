import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _gpu_count() -> int:
    try:
        from onnx_runtime_dart_b200 import _lib
        import ctypes
        n = ctypes.c_int(0)
        rc = _lib.load().ort_cuda_device_count(ctypes.byref(n))
        return n.value if rc == 0 else 0
    except ImportError:
        # The library must exist wherever GPU tests run; without it, GPU tests
        # fail loudly at import rather than being skipped.
        return -1


def pytest_collection_modifyitems(config, items):
    n = None
    for item in items:
        if "gpu" in item.keywords:
            if n is None:
                n = _gpu_count()
            if n == 0:
                item.add_marker(pytest.mark.skip(reason="no CUDA device visible"))


@pytest.fixture(scope="session")
def golden():
    """Loads tests/golden/<case>.npz (extracted from the reference's
    test/fixtures by tests/golden/make_golden.py)."""
    import json
    import numpy as np

    def load(case):
        z = np.load(os.path.join(ROOT, "tests", "golden", case + ".npz"))
        d = {k: z[k] for k in z.files if k != "meta"}
        d["meta"] = json.loads(str(z["meta"]))
        return d
    return load


def max_rel(ref, got):
    """max|dY| / max|Y_ref| (fixture_parity_test.dart:242 style)."""
    import numpy as np
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    den = np.abs(ref).max() if ref.size else 0.0
    d = np.abs(ref - got).max() if ref.size else 0.0
    return float(d / den) if den > 0 else float(d)


def cosine(ref, got):
    import numpy as np
    ref = np.asarray(ref, np.float64).ravel()
    got = np.asarray(got, np.float64).ravel()
    return float(ref @ got / (np.linalg.norm(ref) * np.linalg.norm(got)))
