import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def load_package():
    name = "inference_cpp_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "inference.cpp_b200")
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    name = "ib_oracle"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "oracle", "oracle.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def ib():
    return load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    return load_oracle()


@pytest.fixture(scope="session")
def port(oracle_mod):
    return oracle_mod.Port()


@pytest.fixture(scope="session")
def ref(oracle_mod):
    if not oracle_mod.Ref.available():
        pytest.skip("reference oracle (oracle/_ref) not built here")
    return oracle_mod.Ref()


@pytest.fixture(scope="session")
def cuda(ib):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ib.init(0)
    return torch
