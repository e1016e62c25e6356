import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def golden_routing():
    return np.load(os.path.join(GOLDEN, "routing.npz"))


@pytest.fixture(scope="session")
def golden_outputs():
    return np.load(os.path.join(GOLDEN, "outputs.npz"))


@pytest.fixture(scope="session")
def golden_sampled():
    return np.load(os.path.join(GOLDEN, "sampled_rows.npz"))


@pytest.fixture(scope="session")
def cpu_weights():
    """All 32 local experts (offset 0), quantised on the CPU from their seeds."""
    from flashinfer_b200 import workload as wl
    return wl.local_weights(32, 0)


@pytest.fixture(scope="session")
def gpu_weights(cpu_weights):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return tuple(t.to("cuda:0") for t in cpu_weights)


def oracle_weights_for(cpu_weights, experts):
    """uint8/fp32 numpy views of the given local experts' quantised weights."""
    import torch
    w1, s1, w2, s2 = cpu_weights
    W1 = {e: w1[e].view(torch.uint8).numpy() for e in experts}
    W2 = {e: w2[e].view(torch.uint8).numpy() for e in experts}
    return W1, s1.numpy(), W2, s2.numpy()


def bank_weights_for(experts):
    """uint8/fp32 numpy views of the given GLOBAL experts' quantised weights (seeded per expert),
    keyed by global expert id: the oracle's weight dicts for a local range starting at 0."""
    import torch
    from flashinfer_b200 import workload as wl
    W1, S1, W2, S2 = {}, {}, {}, {}
    for e in experts:
        q1, s1, q2, s2 = wl.WeightBank.get(int(e))
        W1[e], W2[e] = q1.view(torch.uint8).numpy(), q2.view(torch.uint8).numpy()
        S1[e], S2[e] = s1.numpy(), s2.numpy()
    return W1, S1, W2, S2
