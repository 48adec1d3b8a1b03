"""Shared fixtures.  `-m gpu` tests need a B200 and the built CUDA library;
everything else runs on the CPU (oracle, file format, ABI surface, host logic)."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libtorchless_b200.so")


# Seeds/configs of the golden models (tests/golden/make_golden.py: MODELS).
GOLDEN_MODELS = {"tiny": ("TINY", 7), "small": ("SMALL", 3)}


@pytest.fixture(scope="session")
def golden_expected():
    with open(os.path.join(GOLDEN, "reference_expected.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def export_hashes():
    with open(os.path.join(GOLDEN, "export_hashes.json")) as f:
        return json.load(f)


def golden_greedy(name: str):
    d = np.load(os.path.join(GOLDEN, f"ref_greedy_{name}.npz"))
    return d["prompt"].tolist(), d["ids"].tolist(), d["logits"]


def model_bytes(name: str) -> np.ndarray:
    """The seeded golden model binary (numpy exporter, byte-identical to export_mistral.py)."""
    from torchless_b200 import synthetic as S
    cfg_name, seed = GOLDEN_MODELS[name]
    return S.make_numpy_model(getattr(S, cfg_name), seed=seed, norm="random").buf


@pytest.fixture(scope="session")
def tiny_bin():
    return model_bytes("tiny")


@pytest.fixture(scope="session")
def small_bin():
    return model_bytes("small")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    return oracle.oracle_lib()


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """max |a - b| / max |b| (the logits parity metric)."""
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))
