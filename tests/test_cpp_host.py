"""The C++ host mirror (include/moe_b200.hpp) compiles against the C ABI, and
on a GPU its Moe::run matches the CPU restatement (tests/cpp/host_mirror_test.cpp)."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "cpp" / "host_mirror_test.cpp"
LIBDIR = ROOT / "open_rknpu2_lm_infer_b200"


def compile_test(out: Path):
    from oracle import oracle as O
    O.build()
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", str(SRC), "-o", str(out),
           f"-L{LIBDIR}", "-lmoe_b200", f"-Wl,-rpath,{LIBDIR}",
           f"-L{ROOT / 'oracle'}", "-l:libmoe_oracle.so", f"-Wl,-rpath,{ROOT / 'oracle'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_cpp_host_mirror_compiles(tmp_path):
    compile_test(tmp_path / "host_mirror_test")


@pytest.mark.gpu
def test_cpp_host_mirror_runs(cuda, tmp_path):
    exe = tmp_path / "host_mirror_test"
    compile_test(exe)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
