"""The C-ABI library loads on a machine without a GPU and exports every
entry point that include/mars_b200.h declares (no compute calls here)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mars_b200.h")
LIB = os.path.join(ROOT, "cuda-multimodal-memory_b200", "lib", "libmars_b200.so")


def declared_functions(path=HEADER):
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mars_[a-z0-9_]+)\s*\(", text)))


def dynamic_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_library_built():
    assert os.path.exists(LIB), "run make -C cuda-multimodal-memory_b200"


def test_library_loads_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.mars_abi_version.restype = ctypes.c_int
    assert lib.mars_abi_version() == 1
    lib.mars_status_string.restype = ctypes.c_char_p
    assert lib.mars_status_string(4) == b"capacity exceeded"


def test_every_declared_function_is_exported():
    decl = declared_functions()
    assert len(decl) >= 20
    syms = dynamic_symbols(LIB)
    missing = [f for f in decl if f not in syms]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_the_abi():
    import mars_b200
    bound = set(mars_b200.exported_symbols())
    missing = [f for f in declared_functions() if f not in bound]
    assert not missing, f"not bound in mars_b200: {missing}"


def test_calls_fail_cleanly_without_a_device():
    import mars_b200
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    with pytest.raises(mars_b200.MarsError) as e:
        mars_b200.Store(16, 8)
    assert e.value.status in (mars_b200.MARS_ERR_NO_DEVICE, mars_b200.MARS_ERR_CUDA)


def test_python_limits_match_the_header():
    import mars_b200
    text = open(HEADER).read()
    defines = {m.group(1): int(m.group(2))
               for m in re.finditer(r"#define\s+(MARS_[A-Z0-9_]+)\s+(\d+)", text)}
    assert mars_b200.MAX_TOP_K == defines["MARS_MAX_TOP_K"]
    assert mars_b200.NOALLOC_MAX_K == defines["MARS_NOALLOC_MAX_K"]
    assert mars_b200.MAX_BFS_HOPS == defines["MARS_MAX_BFS_HOPS"]
