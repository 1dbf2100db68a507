"""Builds the C++ host API's test programs (tests/cpp/*.cpp) with g++ for
the tests: C++17, every warning an error, linked against the in-tree
library, the CPU stand-in of its C ABI, or the oracle (the checker)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
CPP = REPO / "tests" / "cpp"
LIB_DIR = REPO / "ultravec-ann_b200"
CUDA_LIB = Path("/usr/local/cuda/lib64")
ORACLE_DIR = REPO / "oracle"


def build(out_dir: Path, name: str, sources, link_library: bool, link_oracle: bool = False,
          extra_flags=()) -> Path:
    gxx = shutil.which("g++")
    assert gxx is not None, "g++ is needed to build the C++ host API's tests"
    exe = Path(out_dir) / name
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", f"-I{REPO / 'include'}",
           f"-I{CPP}", *extra_flags, *[str(CPP / s) for s in sources], "-o", str(exe)]
    if link_library:
        assert (LIB_DIR / "libultravec_b200.so").exists(), "build the library first"
        cmd += [f"-L{LIB_DIR}", "-lultravec_b200", f"-Wl,-rpath,{LIB_DIR}", f"-L{CUDA_LIB}",
                f"-Wl,-rpath,{CUDA_LIB}"]
    if link_oracle:
        assert (ORACLE_DIR / "liboracle_uv.so").exists(), "build the oracle first"
        cmd += [f"-I{ORACLE_DIR}", f"-L{ORACLE_DIR}", "-loracle_uv", f"-Wl,-rpath,{ORACLE_DIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-4000:]
    return exe


def run(exe: Path, *args, timeout: int = 300) -> str:
    r = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True,
                       timeout=timeout)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    return r.stdout
