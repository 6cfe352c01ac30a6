"""Drop-in layout details of the reference's C++ API (include/memory_cuda.cuh):
a caller compiled against this repository's headers may name the reference's
QueryContext members, and DeviceMemoryGraph::d_embeddings holds the rows as
the reference lays them out (dense N x D) also when D % 4 != 0
(tests/compat_layout.cpp, compiled here with g++ and linked with the
library)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "cuda-multimodal-memory_b200", "lib")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_reference_layout_caller(tmp_path):
    exe = str(tmp_path / "compat_layout")
    build = subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I",
                            os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "compat_layout.cpp"),
                            "-o", exe, "-L", LIBDIR, "-lmars_b200", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                            f"-Wl,-rpath,{LIBDIR}"], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0 and "ok" in run.stdout, run.stdout + run.stderr
