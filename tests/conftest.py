"""Shared fixtures: paths, the oracle, the reference build, golden fixtures.

Markers: ``gpu`` -- needs an sm_100 GPU; everything else runs on CPU.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen38-in-c_b200")
for p in (PKG, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden"), os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def orc():
    import oracle

    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle

    if not oracle.Reference.available():
        pytest.skip("oracle/_ref/libq35ref.so not built (reference tree absent at build time)")
    return oracle.Reference()


@pytest.fixture(scope="session")
def golden():
    """The reference's 8 matmul known-answer cases, regenerated and pinned."""
    import mm_fixtures as M

    data = M.generate()
    pins = M.pins()
    for name, files in data.items():
        for ext, b in files.items():
            key = f"{name}.{ext}"
            if key in pins["files"] and ext != "yref":
                assert M.sha256(b) == pins["files"][key], f"regenerated {key} differs from the reference's"
        assert M.yref_f32_digest(files["yref"]) == pins["yref_f32"][name], f"{name}.yref differs"
    return {name: M.load_case(files, name) for name, files in data.items()}


@pytest.fixture(scope="session")
def lib():
    import q35cu

    return q35cu.load()


@pytest.fixture(scope="session")
def gpu(lib):
    """A usable sm_100 device for the C-ABI; GPU tests fail loudly without the library."""
    import q35cu

    if lib.q35cu_device_count() <= 0:
        pytest.skip("no CUDA device")
    q35cu.check(lib.q35cu_set_device(0))
    lib.q35cu_set_error_mode(q35cu.ON_ERROR_RECORD)
    yield lib
    lib.q35cu_release_all()


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)
