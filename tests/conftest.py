"""Shared fixtures. Tests marked ``gpu`` need a B200 and the built native library."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built card_playing_gym_b200 native library")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {key: data[key] for key in data.files}


def trunk_fixture(name: str) -> tuple[dict, dict]:
    """(fixture arrays, model config dict) for tests/golden/trunk_<name>.npz."""

    data = load_golden(f"trunk_{name}")
    config = {}
    for key, value in zip(data["config_keys"], data["config_values"]):
        key, value = str(key), str(value)
        config[key] = value if key == "value_embeddings" else int(value)
    return data, config


@pytest.fixture(scope="session")
def golden():
    return load_golden
