import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "1188b-reference-kernels_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(PKG), str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full reference-shape check (tens of seconds)")


_cache = {}


def load_golden(name: str):
    if name not in _cache:
        with np.load(GOLDEN / name, allow_pickle=False) as z:
            _cache[name] = {k: z[k] for k in z.files}
    return _cache[name]


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import moe_b200
    moe_b200.load_library()  # loud failure if the extension is missing
    return torch.device("cuda", 0)


def load_bundle(case_dir: str):
    """Imports 1188b-reference-kernels_b200/bundles/<case_dir>/kernel.py under a unique name."""
    import importlib.util
    path = PKG / "bundles" / case_dir / "kernel.py"
    name = f"bundle_{case_dir}"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def u16(t):
    """bf16 torch tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().contiguous().cpu().view(__import__("torch").int16).numpy().view(np.uint16)


def from_u16(a, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
