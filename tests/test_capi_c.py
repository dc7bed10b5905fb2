"""The C ABI from plain C (CPU): tests/c/abi_smoke.c is compiled with gcc against
include/b200_attn.h alone, linked to libb200attn.so and run."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "learn-nano-vllm_b200")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_caller(tmp_path, pkg):
    pkg.lib()  # built and loadable
    exe = tmp_path / "abi_smoke"
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_smoke.c"), "-L", PKG, "-l:libb200attn.so",
           f"-Wl,-rpath,{PKG}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.startswith("ok abi"), r.stdout + r.stderr
