import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size parity cases")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("GPU tests need a CUDA device (this library has no CPU path)")
    import cti_b200  # noqa: F401  (fails loudly if the library is missing)

    return torch.device("cuda", 0)
