"""The C ABI from a plain C program (gcc, no Python, no torch): the binding a
C host of the reference would use."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mlir-flashattention_b200")


def _build(tmp_path, pkg):
    pkg.lib()  # the library exists
    exe = str(tmp_path / "attn_c_host")
    subprocess.run(
        ["gcc", "-O1", "-std=c11", os.path.join(ROOT, "tests", "c_host", "attn_c_host.c"),
         "-I", os.path.join(ROOT, "include"), "-L", PKG, "-lattnrt", f"-Wl,-rpath,{PKG}", "-lm",
         "-o", exe], check=True)
    return exe


def test_c_host_builds_and_fails_loudly_without_gpu(tmp_path, pkg):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    exe = _build(tmp_path, pkg)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 2 and "no sm_100 device" in r.stdout, r.stdout


@pytest.mark.gpu
def test_c_host_runs_on_gpu(tmp_path, pkg):
    exe = _build(tmp_path, pkg)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "max_rel_err" in r.stdout
