import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")


def load_golden(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def golden_cases(prefix="case_"):
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".pt"))


@pytest.fixture(scope="session", autouse=True)
def _cpu_threads():
    previous = torch.get_num_threads()
    torch.set_num_threads(min(previous, 4))
    yield
    torch.set_num_threads(previous)
