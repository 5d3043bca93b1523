"""The C ABI from a plain C11 host (tests/c_host/dcn_c_host.c): the program a Swift or other
C-ABI caller would write, with device memory from the CUDA runtime and no Python or torch in
the process.  Without a GPU it must compile and link against include/dcn_b200.h and the built
library (the header is plain C); on a B200 it runs the FP16 operator on both tensor-core paths,
the bit-exact FP32 path, the temporal preparation (both its forms, bit-exact), the non-finite flag
and the error codes against the C oracle."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
SRC = REPO / "tests" / "c_host" / "dcn_c_host.c"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _build(tmp_path: Path) -> Path:
    import oracle
    from jasnamacos_b200 import _native

    gcc = shutil.which("gcc")
    assert gcc, "gcc is needed to build the C host"
    lib = _native.LIB_PATH
    assert lib.exists(), "build the library first (python -m jasnamacos_b200.csrc.build)"
    oracle_lib = oracle.build()
    exe = tmp_path / "dcn_c_host"
    cmd = [gcc, "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{REPO / 'include'}", f"-I{REPO / 'oracle'}",
           f"-I{CUDA / 'include'}", str(SRC), "-o", str(exe), f"-L{lib.parent}", "-ldcn_b200",
           f"-L{oracle_lib.parent}", "-ldcn_oracle", f"-L{CUDA / 'lib64'}", "-lcudart", "-lm",
           f"-Wl,-rpath,{lib.parent}:{oracle_lib.parent}:{CUDA / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


def test_c_host_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
def test_c_host_runs_on_the_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("PASS"), r.stdout + r.stderr
