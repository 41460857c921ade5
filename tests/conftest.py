import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG_DIR = os.path.join(ROOT, "jammi-ai_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# A checkout of the reference (f-inverse/jammi-ai), where one exists: the
# tests that re-read its own fixtures (weights, tokenizer files) run only
# when JAMMI_REFERENCE names it, and skip otherwise.
REFERENCE = os.environ.get("JAMMI_REFERENCE", "")


def reference_path(*parts):
    """A file inside the reference checkout, or "" when none is configured."""
    return os.path.join(REFERENCE, *parts) if REFERENCE else ""


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_golden(name):
    import numpy as np
    z = np.load(os.path.join(GOLDEN, name))
    weights = {k[3:]: z[k] for k in z.files if k.startswith("w::")}
    rest = {k: z[k] for k in z.files if not k.startswith("w::")}
    return weights, rest


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
