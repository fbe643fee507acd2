"""pytest configuration: the `gpu` marker and loaders for the package and the oracle.

The package directory is named ``parakeet.cpp_b200`` (not a valid module name),
so it is loaded by path and registered as ``parakeet_b200``.
"""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "parakeet.cpp_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")


def _load(name, path, pkg_dir=None):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [pkg_dir]} if pkg_dir else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_pkg():
    return _load("parakeet_b200", os.path.join(PKG_DIR, "__init__.py"), PKG_DIR)


def load_oracle():
    load_pkg()
    return _load("pk_oracle", os.path.join(ORACLE_DIR, "oracle.py"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pk():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    return load_oracle()
