"""CPU: the C++ host layer (candle-3d_b200/host/candle_l3d.hpp) compiles
against the C ABI header and passes its host-side checks
(tests/host_cpp/test_candle_host.cpp): Layout algebra of the strided head
views, descriptors, the checks that throw before allocation, and the
library's own status codes surfacing as l3d::candle::Error."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_cpp_host_layer(pkg, tmp_path):
    lib = pkg._lib.LIB_PATH
    exe = tmp_path / "test_candle_host"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT / 'candle-3d_b200' / 'host'}", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           str(ROOT / "tests" / "host_cpp" / "test_candle_host.cpp"), "-o", str(exe),
           f"-L{CUDA / 'lib64'}", "-lcudart", str(lib),
           f"-Wl,-rpath,{lib.parent}", f"-Wl,-rpath,{CUDA / 'lib64'}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ALL OK"), r.stdout
