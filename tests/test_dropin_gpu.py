"""A ThunderKittens-SM7x-style C++ caller compiles unchanged against include/ and
runs against libtk_b200.so (the drop-in boundary, exercised from C++)."""

import os
import subprocess

import pytest

import tk_b200

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_cpp_dropin_caller(tmp_path):
    exe = tmp_path / "dropin"
    lib_dir = os.path.dirname(tk_b200.LIB_PATH)
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "dropin", "dropin_main.cu"), "-o", str(exe), "-L", lib_dir,
                    "-ltk_b200", f"-Xlinker=-rpath={lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "drop-in: PASS" in out.stdout
