"""Shared fixtures.  `-m "not gpu"` runs here on CPU; `-m gpu` needs a B200."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__ as ge  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def pkg():
    return ge.load_package()


@pytest.fixture(scope="session")
def synth():
    return ge.load_synth()


@pytest.fixture(scope="session")
def checker():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def tiny_files(tmp_path_factory, synth):
    """Tiny-model GGUFs: f32 weights and bf16-rounded weights, both norm inits."""
    d = tmp_path_factory.mktemp("gguf")
    cfg = dict(synth.TINY)
    out = {}
    for w in ("f32", "bf16"):
        for norm in ("normal", "one_plus"):
            out[(w, norm)] = synth.write_gguf(d / f"tiny_{w}_{norm}.gguf", cfg, seed=0, weights=w, norm_init=norm)
    return cfg, out


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """max |a - b| / max |b|: the relative logit deviation used by the parity bars."""
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(float(np.max(np.abs(b))), 1e-30))
