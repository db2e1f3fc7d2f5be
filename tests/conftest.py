"""Shared fixtures. GPU tests carry @pytest.mark.gpu; `-m "not gpu"` runs the rest on the CPU."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_golden.npz"

SMALL = {"d_model": 128, "num_layers": 3, "n_heads": 4, "kv_heads": 2, "qk_ratio": [0.25, 0.5, 0.75], "mlp_hidden": 320, "value_bins": 16}
TINY = {"d_model": 256, "num_layers": 6, "n_heads": 8, "kv_heads": 4, "qk_ratio": [0.25, 0.5, 0.75] * 2, "mlp_hidden": 1024,
        "value_bins": 128}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)
