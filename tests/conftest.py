"""Shared test setup: the `gpu` marker, the oracle import path and the product package loader."""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
# The reference checkout (a directory named reference beside this repository, or LJX_REFERENCE)
# is only present where the fixtures were made; tests that need its data files (the CuZr table)
# skip elsewhere.
REFERENCE = Path(os.environ.get("LJX_REFERENCE", ROOT.parent / "reference"))
CUZR_TABLE = REFERENCE / "examples" / "potentials" / "CuZr.eam.alloy.gz"

sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")


def load_package():
    """Import the product package from its hyphenated directory as `lammps_jax_b200`."""
    name = "lammps_jax_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = ROOT / "lammps-jax_b200"
    spec = importlib.util.spec_from_file_location(
        name, pkg_dir / "__init__.py", submodule_search_locations=[str(pkg_dir)])
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


@pytest.fixture(scope="session")
def ljx():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc  # noqa: PLC0415
    orc.lib()
    return orc


def golden(name: str):
    return np.load(GOLDEN / name, allow_pickle=False)
