import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")
    config.addinivalue_line("markers", "slow: long-running")


def load_cases(name: str):
    """Golden cases saved by tests/golden/make_golden.py as c{i}_{key} arrays."""
    import numpy as np
    z = np.load(GOLDEN / name, allow_pickle=False)
    n = int(z["n"])
    cases = []
    for i in range(n):
        pre = f"c{i}_"
        cases.append({k[len(pre):]: z[k] for k in z.files if k.startswith(pre)})
    return cases


def decode_logits(case):
    """Rebuild the logits tensor of an acceptance case in its stored dtype."""
    import numpy as np
    import torch
    lg = case["logits"]
    if str(case["dtype"]) == "bf16":
        return torch.from_numpy(np.ascontiguousarray(lg)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(lg))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs an sm_100 device")
    return torch.device("cuda:0")
