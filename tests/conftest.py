import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "groupgemm-cktile-optimized_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")
    config.addinivalue_line("markers", "slow: large configurations")


def load_package():
    """The product package (its directory name is not a Python identifier)."""
    if "gg_b200" in sys.modules:
        return sys.modules["gg_b200"]
    spec = importlib.util.spec_from_file_location("gg_b200", os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["gg_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if ORACLE_DIR not in sys.path:
        sys.path.insert(0, ORACLE_DIR)
    import oracle  # noqa: E402

    return oracle


def _load_file(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ensure_built():
    if not os.path.exists(os.path.join(PKG_DIR, "lib", "libgg_b200.so")):
        _load_file("gg_pkg_build", os.path.join(PKG_DIR, "build.py")).build()
    if not os.path.exists(os.path.join(ORACLE_DIR, "lib", "liboracle.so")):
        _load_file("gg_oracle_build", os.path.join(ORACLE_DIR, "build.py")).build_oracle()


@pytest.fixture(scope="session")
def gg():
    _ensure_built()
    return load_package()


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    return load_oracle()
