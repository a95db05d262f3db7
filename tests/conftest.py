import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_pkg():
    # The package directory is named `furiosa-opt_b200` (not an identifier), so bind it by path.
    if "furiosa_opt_b200" in sys.modules:
        return sys.modules["furiosa_opt_b200"]
    d = os.path.join(ROOT, "furiosa-opt_b200")
    spec = importlib.util.spec_from_file_location("furiosa_opt_b200", os.path.join(d, "__init__.py"),
                                                  submodule_search_locations=[d])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["furiosa_opt_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_load_pkg()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def b200():
    import furiosa_opt_b200 as fb
    return fb.B200(0)
