import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built sm_100a library")


@pytest.fixture(scope="session")
def layout_golden():
    return np.load(os.path.join(GOLDEN, "layout_golden.npz"))


@pytest.fixture(scope="session")
def ops_golden():
    return np.load(os.path.join(GOLDEN, "ops_golden.npz"))


def op_case(z, name):
    """Unpack one ops_golden case into plain numpy/python objects."""
    p = name + "/"
    ids = [int(i) for i in z[p + "adapter_ids"]]
    ranks = {i: int(r) for i, r in zip(ids, z[p + "ranks"])}
    alphas = {i: float(a) for i, a in zip(ids, z[p + "alphas"])}
    case = {
        "x": z[p + "x"], "w": z[p + "w"], "g": z[p + "g"],
        "routes": [tuple(int(v) for v in r) for r in z[p + "routes"]],
        "a": {i: z[p + f"a{i}"] for i in ids}, "b": {i: z[p + f"b{i}"] for i in ids},
        "ranks": ranks, "alphas": alphas, "scaling": {i: alphas[i] / ranks[i] for i in ids},
        "y": z[p + "y"], "gx": z[p + "gx"],
        "grad_keys": [int(k) for k in z[p + "grad_keys"]],
        "bf16": bool(z[p + "bf16"]),
    }
    case["ga"] = {k: z[p + f"ga{k}"] for k in case["grad_keys"]}
    case["gb"] = {k: z[p + f"gb{k}"] for k in case["grad_keys"]}
    return case
