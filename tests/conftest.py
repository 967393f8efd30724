import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "hxq-native_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _ensure_built():
    lib = os.path.join(PKG, "lib", "libhxq.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    orc = os.path.join(REPO, "oracle", "liboracle.so")
    if not os.path.exists(orc):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def H():
    _ensure_built()
    import hxq_b200
    hxq_b200.lib()
    return hxq_b200


@pytest.fixture(scope="session")
def L(H):
    return H.lib()


@pytest.fixture(scope="session")
def oracle():
    _ensure_built()
    from oracle.oracle import Oracle
    return Oracle()


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {}
    for k in z.files:
        v = z[k]
        if k.startswith("meta_"):
            d[k[5:]] = v.item()
        else:
            d[k] = v
    return d


def golden_names(prefix: str = "") -> list[str]:
    """Fixtures of the reference library (hxq.c, hxq_affine.c) whose names
    start with `prefix`; the container converter's fixtures (container_*)
    only when asked for by that prefix."""
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz") and f.startswith(prefix)
                  and (prefix.startswith("container") or not f.startswith("container")))


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device; GPU tests fail (not skip) without one."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    torch.cuda.init()
    return torch
