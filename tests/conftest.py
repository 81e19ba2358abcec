import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "diffuse-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: builds full-size (GB) synthetic layers")


def _ensure_built():
    lib = os.path.join(PKG, "libdiffuse_moe.so")
    syn = os.path.join(PKG, "libdmoe_synth.so")
    orc = os.path.join(ORACLE, "libdmoe_oracle.so")
    if not (os.path.exists(lib) and os.path.exists(syn)):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    if not os.path.exists(orc):
        subprocess.run(["make", "-s", "-C", ORACLE], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def gpu_available():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
