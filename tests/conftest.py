import os
import sys
import warnings

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    for line in (
        "gpu: needs a CUDA device (sm_100a) and the built libcg_b200.so",
        "slow: large shapes or many processes",
        "ddp: spawns processes (gloo on CPU, NCCL on GPUs)",
        "compiled: region-plan behaviour (kept for parity with the reference's markers)",
    ):
        config.addinivalue_line("markers", line)


@pytest.fixture(autouse=True)
def _fresh_region_state():
    import create_graph_b200 as cg

    cg.reset()
    warnings.filterwarnings("ignore", message=".*TensorFloat32.*")
    yield
    cg.reset()


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs CUDA")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
