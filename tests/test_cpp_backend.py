"""The reference's C++ CudaTest cases run through the inference::cuda mirror
(include/ib_cuda_backend.hpp), built with g++ against libib_cuda.so."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "backend_test.cpp")
LIBDIR = os.path.join(ROOT, "inference.cpp_b200")


def _build(tmp_path, ib):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path / "backend_test")
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           SRC, "-L", LIBDIR, "-lib_cuda", "-Wl,-rpath," + LIBDIR, "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_shim_compiles_and_links(tmp_path, ib):
    exe = _build(tmp_path, ib)
    assert os.path.exists(exe)


def test_shim_exports_reference_names(ib):
    """Every function of the reference's inference::cuda namespace is exported."""
    r = subprocess.run(["nm", "-D", "--defined-only", "-C", os.path.join(LIBDIR, "libib_cuda.so")],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.skip("nm not available")
    names = {"available", "device_name", "total_memory", "free_memory", "sync", "shutdown",
             "alloc", "release", "upload", "download", "gemv", "gemv_i16", "gemm", "gemm_i16",
             "rmsnorm", "silu", "mul", "add", "embedding", "embedding_i16", "embedding_batch",
             "embedding_batch_i16", "kv_write", "kv_write_batch", "rope", "rope_batch",
             "attention", "attention_batch"}
    exported = set()
    for line in r.stdout.splitlines():
        if "inference::cuda::" in line:
            exported.add(line.split("inference::cuda::", 1)[1].split("(", 1)[0].split("[", 1)[0])
    assert names <= exported, sorted(names - exported)


@pytest.mark.gpu
def test_reference_cuda_cases(tmp_path, ib, cuda):
    exe = _build(tmp_path, ib)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout
