"""Shared fixtures and the `gpu` marker.

`-m "not gpu"` runs here on the CPU: the oracle against the reference's golden vectors, host
logic, and the C-ABI library's exports. `-m gpu` runs on a B200 and checks the CUDA path against
the oracle through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name: str) -> dict[str, np.ndarray]:
    path = GOLDEN / f"golden_{name}.npz"
    if not path.exists():
        pytest.skip(f"{path.name} not generated")
    return dict(np.load(path, allow_pickle=False))


def case_bundle(case: str):
    """The seeded bundle a golden case was made from (make_golden.CASES)."""
    from make_golden import CASES

    from so101_smolvla_edge_b200.bundle import seeded_bundle
    from so101_smolvla_edge_b200.spec import ModelSpec

    kw, repr_, hw = CASES[case]
    return seeded_bundle(ModelSpec(**kw), seed=7, action_repr=repr_, image_hw=hw, state_dim=6,
                         action_dim=6, style="test")  # fmt: skip


_CONFIG0 = {}


def config0_bundle():
    """BASELINE configs[0], built once per session (~2 s)."""
    if "b" not in _CONFIG0:
        from so101_smolvla_edge_b200.bundle import seeded_bundle

        _CONFIG0["b"] = seeded_bundle()
    return _CONFIG0["b"]
