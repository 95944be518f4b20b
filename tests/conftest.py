"""pytest setup: the `gpu` marker, import paths for the oracle and the package.

The package directory is `web-engine_b200/` (not an importable identifier), so it is
loaded under the module name `web_engine_b200`.
"""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    if "web_engine_b200" in sys.modules:
        return sys.modules["web_engine_b200"]
    pkg_dir = os.path.join(ROOT, "web-engine_b200")
    spec = importlib.util.spec_from_file_location(
        "web_engine_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["web_engine_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the C-ABI library on cuda:0)")


@pytest.fixture(scope="session")
def we():
    return load_package()


@pytest.fixture(scope="session")
def graph(we):
    """One library context on cuda:0 for the GPU tests."""
    g = we.Graph(0)
    yield g
    g.destroy()
