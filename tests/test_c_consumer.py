"""The C ABI from a plain C99 program (tests/c_consumer.c): the header compiles
as C with warnings as errors, the program links libhilberta_b200.so and its
host-side calls behave (no GPU needed)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_program_uses_the_abi(tmp_path):
    from hilberta_b200 import build

    so = build.build()
    exe = tmp_path / "c_consumer"
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "c_consumer.c"), "-o", str(exe), "-L", str(so.parent), "-lhilberta_b200",
           f"-Wl,-rpath,{so.parent}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    assert run.stdout.strip() == "ok"
