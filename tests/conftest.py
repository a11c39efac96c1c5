"""Shared fixtures.  Tests marked ``gpu`` need a CUDA device (a B200); the
rest run on any CPU and cover the oracle, the host logic and the library
boundary."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_fixtures.npz"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.fixture(scope="session")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def tiny_state(golden: dict[str, np.ndarray], which: str) -> dict[str, np.ndarray]:
    pre = which + "/"
    return {k[len(pre):]: v for k, v in golden.items() if k.startswith(pre)}


def tiny_dims(golden: dict[str, np.ndarray], which: str):  # -> oracle.model.Dims
    from oracle.model import Dims

    v, L, d, h, hkv, ff, msl = (int(x) for x in golden[f"{which}_cfg"])
    return Dims(vocab_size=v, d_model=d, n_layers=L, n_heads=h, n_kv_heads=hkv, d_ff=ff,
                max_seq_len=msl)
