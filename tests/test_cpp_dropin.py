"""The C++ mirror (include/hkv_hashtable.h) compiles and links like the
reference's header (CPU), and a program written against npu::hkv::HashTable
runs on the GPU (gpu)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "hkv_cpp_dropin.cpp")
PKG = os.path.join(ROOT, "hierarchicalkv-ascend_b200")
CUDA = "/usr/local/cuda"


def build(out):
    cmd = ["g++", "-std=c++17", "-O1", SRC, "-o", out, f"-I{ROOT}/include",
           f"-I{CUDA}/include", f"-L{PKG}", "-l:libhkv_b200.so", f"-Wl,-rpath,{PKG}",
           f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


SCAN_SRC = os.path.join(ROOT, "tests", "cpp", "hkv_scan_dropin.cu")


def build_scan(out):
    """nvcc translation unit using the functor scans (hkv_scan.cuh)."""
    cmd = [f"{CUDA}/bin/nvcc", "-std=c++17", "-O1",
           "-gencode", "arch=compute_100a,code=sm_100a", SCAN_SRC, "-o", out,
           f"-I{ROOT}/include", f"-L{PKG}", "-l:libhkv_b200.so",
           "-Xlinker", f"-rpath={PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def test_scan_templates_compile_with_nvcc(tmp_path):
    build_scan(str(tmp_path / "scan"))
    assert os.path.exists(tmp_path / "scan")


@pytest.mark.gpu
def test_scan_templates_run(tmp_path):
    exe = str(tmp_path / "scan")
    build_scan(exe)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "cpp scan drop-in ok" in r.stdout


def test_cpp_mirror_compiles_and_links(tmp_path):
    build(str(tmp_path / "dropin"))
    assert os.path.exists(tmp_path / "dropin")


@pytest.mark.gpu
def test_cpp_mirror_runs(tmp_path):
    exe = str(tmp_path / "dropin")
    build(exe)
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "cpp drop-in ok" in r.stdout
