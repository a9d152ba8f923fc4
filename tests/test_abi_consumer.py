"""The C ABI from compiled host code: tests/abi_consumer.c is built as C99 and as C++14 against
include/sam3_b200.h and linked with libsam3_b200.so, then run (host-only checks; no GPU needed)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sam3.cpp_b200")


@pytest.mark.parametrize("compiler,flags", [("gcc", ["-std=c99"]), ("g++", ["-std=c++14", "-x", "c++"])])
def test_header_and_library_from_c_and_cpp(b200, tmp_path, compiler, flags):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not installed")
    b200.lib()  # fails loudly if the library was not built
    exe = str(tmp_path / "abi_consumer")
    subprocess.run([compiler, *flags, "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "abi_consumer.c"), "-L", PKG, "-lsam3_b200",
                    f"-Wl,-rpath,{PKG}", "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
