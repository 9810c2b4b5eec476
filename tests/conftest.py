import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU reference comparison")


@pytest.fixture(scope="session")
def golden_cases():
    return np.load(GOLDEN / "ame_cases.npz")


@pytest.fixture(scope="session")
def config1_golden():
    return np.load(GOLDEN / "config1_exact.npz")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import n550_qwen3_bringup_handover_b200 as n5
    n5.lib()
    return torch.device("cuda:0")


def to_dev_bf16(a: np.ndarray, device):
    """uint16 BF16 bit pattern array -> torch.bfloat16 tensor on device."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16))
    return t.view(torch.bfloat16).to(device)


def bf16_bits(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def case_operands(z, cid):
    """(A bf16 bits [M, lda], B bf16 bits [N, ldb], M, N, K, lda, ldb, a_src or None)."""
    import oracle
    M, N, K, lda, ldb, mixed = (int(v) for v in z[f"{cid}/shape"])
    a_src = None
    if mixed:
        a_src = z[f"{cid}/a_src"]
        a = oracle.f32_to_bf16(a_src)
    else:
        a = z[f"{cid}/a"]
    return a, z[f"{cid}/b"], M, N, K, lda, ldb, a_src
