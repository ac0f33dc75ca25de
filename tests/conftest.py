import hashlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Parity bar of the path: attention outputs within max-abs 2e-3 and rel 1e-2
# of the oracle (|gpu - ref| <= ATOL + RTOL * |ref| elementwise).
ATOL = 2e-3
RTOL = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle as O

    if not os.path.exists(O.ORACLE_SO):
        O.build(with_ref=False)
    O.lib()
    return O


def golden(name):
    return np.load(os.path.join(ROOT, "tests", "golden", name))


def digest(arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).view(np.uint8).tobytes())
    return h.hexdigest()


def assert_close(got, ref, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside tolerance, max abs err "
                           f"{float(err.max()):.3e}")
