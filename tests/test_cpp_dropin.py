"""The C++ drop-in (include/neural_textures/train.h, forward_pass_test.h).

- The reference driver's own training loop and inference call (mavenkim2/neural_textures
  main.cpp, from the inference-output allocation through the copy of the output back to the
  host, lines 1011-1100), read from a checkout of the reference when one is present, compile
  unchanged against the drop-in header and link with the library (CPU).
- tests/cpp/driver_loop.cpp, a reference-style driver with the same set-up and loop written
  against the header, compiled with g++: without a GPU a rejected call surfaces as
  std::runtime_error; on a B200 it runs the known-answer test, 200 training steps against
  reference textures and inference with the reference's [N][16] fp32 output layout."""
import json
import os
import subprocess
import sys

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


PRELUDE = r"""
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "neural_textures/train.h"

using namespace neural_textures;

static void CheckCuda(cudaError_t e, const char *what)
{
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
template <typename T>
static T *AllocateDeviceBuffer(size_t n, const char *what)
{
    T *p = nullptr;
    CheckCuda(cudaMalloc(&p, n * sizeof(T)), what);
    return p;
}
template <typename T>
static void ZeroDeviceBuffer(T *p, size_t n, const char *what)
{
    CheckCuda(cudaMemset(p, 0, n * sizeof(T)), what);
}

void ReferenceTrainingLoop(KernelParams &params)
{
"""
EPILOGUE = r"""
}

int main()
{
    KernelParams params;
    ReferenceTrainingLoop(params);
    return 0;
}
"""


def _reference_main():
    sys_path = ROOT if ROOT in sys.path else None
    if sys_path is None:
        sys.path.insert(0, ROOT)
    import __graft_entry__
    path = os.path.join(__graft_entry__.REFERENCE_ROOT, "main.cpp")
    return path if os.path.exists(path) else None


def test_reference_driver_loop_compiles_against_dropin(native, tmp_path):
    path = _reference_main()
    if path is None:
        pytest.skip("no checkout of the reference on this host")
    lines = open(path).read().splitlines()
    start = next(i for i, l in enumerate(lines) if "const size_t inferenceSampleCount" in l)
    end = next(i for i, l in enumerate(lines) if '"cudaMemcpy(inferenceOutput)");' in l and i > start)
    body = [l for l in lines[start:end + 1] if l.strip() != "#if 1"]  # its #endif lies past the extract
    assert any("InvokeTraining(params, type);" in l for l in body)
    assert any("InvokeInference(params);" in l for l in body)
    src = tmp_path / "reference_loop.cpp"
    src.write_text(PRELUDE + "\n".join(body) + EPILOGUE)
    from neural_textures_b200 import _native
    libdir = os.path.dirname(_native.LIB_PATH)
    exe = str(tmp_path / "reference_loop")
    cmd = ["g++", "-std=c++17", "-O1", str(src), "-o", exe, "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), "-L", libdir, "-lnt_b200", "-L", os.path.join(CUDA, "lib64"),
           "-lcudart", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


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
    assert d["zero_tail"], d
