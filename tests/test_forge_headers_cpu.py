"""The forge:: C++ headers (include/forge/) are what the reference's callers
include: each one compiles on its own, as `#include "forge/<name>"` with only
the include directory on the path, without warnings (no GPU needed)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FORGE = os.path.join(ROOT, "include", "forge")
HEADERS = sorted(f for f in os.listdir(FORGE) if f.endswith(".hpp"))


@pytest.mark.parametrize("name", HEADERS)
def test_header_compiles_alone(tmp_path, name):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    src = tmp_path / "one.cpp"
    src.write_text(f'#include "forge/{name}"\nint main() {{ return 0; }}\n')
    r = subprocess.run([cxx, "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror",
                        "-I" + os.path.join(ROOT, "include"), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
