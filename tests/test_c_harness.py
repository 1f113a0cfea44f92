"""The C harness (tests/c_harness/ft_harness.c) drives the library through its C
ABI without Python: compiled here with gcc against include/ferris_ternary.h and
the built .so; run on a GPU (marked gpu)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "ferrisres_b200")


def build_harness(out_dir):
    exe = os.path.join(str(out_dir), "ft_harness")
    subprocess.run(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_harness", "ft_harness.c"), "-o", exe,
                    "-L", LIBDIR, "-lferris_ternary", f"-Wl,-rpath,{LIBDIR}", "-lm"], check=True)
    return exe


def test_harness_compiles_and_links(tmp_path):
    assert os.path.exists(build_harness(tmp_path))


@pytest.mark.gpu
def test_harness_runs_on_gpu(tmp_path):
    exe = build_harness(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().endswith("ok")
