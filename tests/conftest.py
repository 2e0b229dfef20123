"""Shared pytest setup: the `gpu` marker, repository paths, fixture loaders."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_small_cases():
    z = np.load(os.path.join(GOLDEN, "small_cases.npz"))
    cases = []
    for i in range(int(z["ncases"])):
        c = {k[len(f"c{i}_"):]: z[k] for k in z.files if k.startswith(f"c{i}_")}
        for key in ("dtype", "bs", "n", "k", "m"):
            c[key] = int(c[key])
        cases.append(c)
    return cases


def load_digests():
    with open(os.path.join(GOLDEN, "config_digests.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def small_cases():
    return load_small_cases()


@pytest.fixture(scope="session")
def digests():
    return load_digests()


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    return oracle.Oracle()


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests skip where there is none (this container)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qraf_b200

    qraf_b200.init(0)
    return torch.device("cuda:0")
