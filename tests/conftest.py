import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gollama.cu_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    # build the in-tree libraries if this checkout has none yet
    if not os.path.exists(os.path.join(PKG, "libgollama_b200.so")):
        subprocess.run(["make", "-C", PKG, "-j8", "-s"], check=True)
    import oracle_lib

    if not os.path.exists(oracle_lib.ORACLE_SO):
        oracle_lib.build()


@pytest.fixture(scope="session")
def gb():
    import gollama_b200

    gollama_b200.lib()
    return gollama_b200


@pytest.fixture(scope="session")
def orc():
    import oracle_lib

    oracle_lib.lib()
    return oracle_lib


@pytest.fixture(scope="session")
def golden():
    import json

    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def kernels(gb, cuda):
    k = gb.Kernels(0)
    yield k
    k.close()
