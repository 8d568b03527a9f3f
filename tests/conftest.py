import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")

# Parity tolerance of the task statement: per-step logits within bf16
# tolerance after fp32 accumulation, and identical greedy tokens wherever the
# reference's top-2 gap exceeds it.
TOL_MAX_ABS = 2e-2
TOL_REL_L2 = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def native_libraries():
    """Build the in-tree native libraries if their sources changed (nvcc
    cross-compiles for sm_100a without a GPU)."""
    from qwen_megakernel_b200.build import build

    return build()


def load_golden(cfg: int) -> dict:
    path = os.path.join(GOLDEN_DIR, f"config{cfg}.npz")
    with np.load(path, allow_pickle=False) as z:
        out = {k: z[k] for k in z.files}
    import json

    out["meta"] = json.loads(str(out["meta"]))
    return out


@pytest.fixture(scope="session")
def golden1():
    return load_golden(1)


@pytest.fixture(scope="session")
def golden2():
    return load_golden(2)


@pytest.fixture(scope="session")
def cuda_weights():
    """Full 28-layer seeded weights on cuda:0 (BASELINE config, seed 0)."""
    import torch

    from qwen_megakernel_b200.weights import random_weights

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return random_weights(seed=0, device="cuda", max_seq_len=2048)
