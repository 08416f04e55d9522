import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"
FORMAT_TAGS = {
    0: "q4_k", 1: "q4_k_split_predecoded", 2: "q4_k_split_half", 3: "q4_k_split_compact",
    4: "q4_k_split_native", 5: "q5_k", 6: "iq2_s", 7: "iq3_s",
}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(fmt: int, case: str) -> dict:
    data = np.load(GOLDEN / f"golden_{FORMAT_TAGS[fmt]}.npz")
    prefix = f"{case}_"
    return {k[len(prefix):]: data[k] for k in data.files if k.startswith(prefix)}


@pytest.fixture(scope="session")
def port():
    import qoracle

    return qoracle.Port()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
