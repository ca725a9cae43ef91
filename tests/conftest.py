"""Shared pytest setup: the ``gpu`` marker and the package loader.

The product package lives in the directory ``gemma-4-omni_b200`` (not a valid
Python identifier); it is loaded under the module name ``gemma4_omni_b200``.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    name = "gemma4_omni_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = ROOT / "gemma-4-omni_b200"
    spec = importlib.util.spec_from_file_location(name, pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built library")


@pytest.fixture(scope="session")
def pkg():
    return load_package()
