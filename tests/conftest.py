"""Shared fixtures.  Tests marked ``gpu`` need a B200 and the built library;
everything else runs on the CPU (oracle, host logic, C-ABI surface)."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))

SMALL = dict(d_model=128, d_kv=64, d_ff=256, num_layers=2, num_heads=2, context_length=512,
             time_encoding_scale=512)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden_small():
    z = np.load(GOLDEN / "small_model.npz")
    cases = {}
    for key in z.files:
        name, field = key.split("/")
        cases.setdefault(name, {})[field] = z[key]
    return cases


@pytest.fixture(scope="session")
def golden_base():
    return dict(np.load(GOLDEN / "base_cfg0.npz"))


@pytest.fixture(scope="session")
def param_names():
    return json.loads((GOLDEN / "param_names.json").read_text())


def small_config(**kw):
    from cutechronos_b200.model import CuteChronos2Config
    d = dict(SMALL)
    d.update(kw)
    return CuteChronos2Config(**d)


def oracle_config(**kw):
    from oracle.chronos2_oracle import OracleConfig
    d = dict(SMALL)
    d.update(kw)
    return OracleConfig(**d)


def case_inputs(c):
    ctx = torch.from_numpy(c["context"])
    mask = torch.from_numpy(c["context_mask"]) if "context_mask" in c else None
    gid = torch.from_numpy(c["group_ids"]) if "group_ids" in c else None
    return ctx, mask, int(c["N"]), gid
