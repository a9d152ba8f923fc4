import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _load_pkg_module(name: str):
    """Load a module from the sam3.cpp_b200/ package directory (its name is
    not a Python identifier, so it is loaded by path)."""
    path = os.path.join(ROOT, "sam3.cpp_b200", f"{name}.py")
    spec = importlib.util.spec_from_file_location(f"sam3_b200_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def b200():
    return _load_pkg_module("b200")


@pytest.fixture(scope="session")
def backend(b200):
    be = b200.Backend(0)
    yield be
    be.free()


@pytest.fixture(scope="session")
def model():
    return _load_pkg_module("model")


def rel_err(got, ref):
    """max |got - ref| / max |ref| -- the normwise form of the north-star
    bound 'fp32 tensor outputs within max relative error 1e-2'."""
    import numpy as np
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.fixture(scope="session")
def ggml_caller(b200, tmp_path_factory):
    """tests/ggml_vit_block.cpp built as C++14 against the ggml-compatible headers and linked with the
    B200 ggml backend (libggml_b200.so) and the ggml core stand-in (libggml_mini.so)."""
    import ctypes
    import shutil
    import subprocess
    if shutil.which("g++") is None:
        pytest.skip("g++ not installed")
    b200.lib()  # fails loudly if the library was not built
    pkg = os.path.join(ROOT, "sam3.cpp_b200")
    for name in ("libggml_b200.so", "libggml_mini.so"):
        if not os.path.exists(os.path.join(pkg, name)):
            raise RuntimeError(f"{name} is not built: run make -C sam3.cpp_b200")
    so = str(tmp_path_factory.mktemp("ggml") / "libggml_vit_block.so")
    subprocess.run(["g++", "-std=c++14", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", "-I",
                    os.path.join(pkg, "ggml"), os.path.join(ROOT, "tests", "ggml_vit_block.cpp"), "-L", pkg,
                    "-lggml_b200", "-lggml_mini", "-lsam3_b200", f"-Wl,-rpath,{pkg}", "-o", so], check=True)
    return ctypes.CDLL(so)
