"""Shared test setup: the `gpu` marker, module loading and build checks."""
import importlib.util
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.5-9b-bfp8b-1xn300_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libqcache.so)")


def load_pkg_module(name):
    """Import a module of the package directory (its name is not an identifier)."""
    full = "qcache_b200_" + name
    if full in sys.modules:
        return sys.modules[full]
    spec = importlib.util.spec_from_file_location(full, os.path.join(PKG, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[full] = mod
    spec.loader.exec_module(mod)
    return mod


def ensure_built():
    if not os.path.exists(os.path.join(PKG, "libqcache.so")):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)


@pytest.fixture(scope="session")
def qcache():
    ensure_built()
    return load_pkg_module("qcache")


@pytest.fixture(scope="session")
def synth():
    return load_pkg_module("synth")


@pytest.fixture(scope="session")
def oracle():
    ensure_built()
    import oracle as o
    return o


@pytest.fixture(autouse=True)
def _release_device_temporaries():
    yield
    mod = sys.modules.get("gpu_util")
    if mod is not None:
        mod.KEEP.clear()
