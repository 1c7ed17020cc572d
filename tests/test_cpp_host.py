"""The C ABI from a compiled C++ host, as the engines use it: a program
(tests/cpp/milda_sequence.cpp) that includes include/b2gguf.h and replays
Milda's call sequence, built with g++ against libb2gguf.so.  It compiles
here; it runs on a GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "arkantos-ai-stack-suite_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "milda_sequence.cpp")


def _build(tmp_path) -> str:
    if not shutil.which("g++"):
        pytest.skip("no g++")
    if not os.path.exists(os.path.join(PKG, "libb2gguf.so")):
        pytest.skip("libb2gguf.so not built")
    exe = str(tmp_path / "milda_sequence")
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    SRC, "-o", exe, "-L", PKG, "-lb2gguf", f"-Wl,-rpath,{PKG}"], check=True)
    return exe


def test_cpp_host_compiles_against_the_header(tmp_path):
    assert os.access(_build(tmp_path), os.X_OK)


@pytest.mark.gpu
def test_cpp_host_replays_milda_sequence(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe, str(tmp_path / "m.gguf")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "milda sequence ok" in r.stdout
    print(r.stdout.strip())
