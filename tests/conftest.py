import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
PKG_DIR = os.path.join(ROOT, "local-llama-pynq-z2_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA device); run with -m gpu")


def load_pkg():
    """Imports the package directory (its name has dashes) as module `mvb`."""
    if "mvb" in sys.modules:
        return sys.modules["mvb"]
    spec = importlib.util.spec_from_file_location("mvb", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mvb"] = mod
    spec.loader.exec_module(mod)
    return mod


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def golden_cases(name):
    """{case: {field: array}} from a fixture whose keys are 'case.field'."""
    z = golden(name)
    out = {}
    for k in z.files:
        case, field = k.split(".", 1)
        out.setdefault(case, {})[field] = z[k]
    return out


@pytest.fixture(scope="session")
def mvb():
    return load_pkg()


@pytest.fixture(scope="session")
def restatement():
    import oracle
    path = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(path):
        import subprocess
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)
    return oracle.Restatement(path)


@pytest.fixture(scope="session")
def data_dir():
    d = os.environ.get("MVB_DATA", "/tmp/mvb_data")
    os.makedirs(d, exist_ok=True)
    return d
