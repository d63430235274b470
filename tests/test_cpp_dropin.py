"""The C++ drop-in (include/neural_textures/train.h, forward_pass_test.h): tests/cpp/driver_loop.cpp
is the reference driver's loop (main.cpp:1037-1091) written against it, compiled with g++ and
linked with the library.  Without a GPU it checks that a rejected call surfaces as
std::runtime_error; on a B200 it runs the known-answer test, 200 training steps and inference."""
import json
import os
import subprocess

import pytest

from tests.conftest import ROOT

CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def driver(native, tmp_path_factory):
    from neural_textures_b200 import _native
    exe = str(tmp_path_factory.mktemp("cpp") / "driver_loop")
    libdir = os.path.dirname(_native.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-O2", os.path.join(ROOT, "tests", "cpp", "driver_loop.cpp"), "-o", exe,
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"), "-L", libdir, "-lnt_b200",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{CUDA}/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_rejected_call_throws(driver):
    r = subprocess.run([driver, "--invalid"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert json.loads(r.stdout.strip().splitlines()[-1])["rejected"]


@pytest.mark.gpu
def test_driver_loop_trains(driver):
    r = subprocess.run([driver, "200"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])  # RunForwardPassTest reports first
    assert d["loss_last"] < 0.5 * d["loss_first"], d
