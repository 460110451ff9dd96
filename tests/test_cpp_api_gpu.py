"""The C++ API (include/da3cpp/da3.h) from a C++ program: tests/cpp/da3_api_check.cpp is
compiled with g++ against the public headers and libda3b.so and run on the GPU. It checks
load_model / model_info / infer, that infer_preprocessed with the reference's upload
callback gives depth and confidence bit-identical to infer on the same image, and the
reference's refusals (DA2 checkpoint on infer_preprocessed, malformed Image), and the DA3
mono and nested metric model kinds through load_model / load_nested_model / infer."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_cpp_api(lib, tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    from da3cpplib_b200 import _lib, synth

    exe = tmp_path / "da3_api_check"
    libdir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-O1", os.path.join(ROOT, "tests", "cpp", "da3_api_check.cpp"), "-I",
           os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"), "-L", libdir, "-l:libda3b.so",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{CUDA}/lib64",
           "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    da3 = synth.ensure_gguf("da3-t", stress=True)
    da2 = synth.ensure_gguf("da2-t", stress=True)
    mono = synth.ensure_gguf("da3m-t", stress=True)
    metric = synth.ensure_gguf("da3m-t", stress=True, metric_branch=True)
    r = subprocess.run([str(exe), da3, da2, "112", mono, metric], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
