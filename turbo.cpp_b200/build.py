"""Builds libturbo_b200.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

Usage: python turbo.cpp_b200/build.py [--force]
The library is rebuilt when a source or header is newer than it.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libturbo_b200.so")
OBJ = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "--expt-relaxed-constexpr"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def build(force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    hdr_time = max(os.path.getmtime(h) for h in headers())
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if (not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time)):
            continue
        cmd = [NVCC] + FLAGS + ["-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out = p.communicate()[0].decode()
        if p.returncode != 0 or verbose:
            sys.stderr.write(out)
        if p.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(failed))
    if force or not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", OUT] + objs
        subprocess.check_call(cmd)
    build_host(force)
    build_selfcheck(force)
    return OUT


SELFCHECK_SRCS = os.path.join(CSRC, "test")
SELFCHECK_OUT = os.path.join(HERE, "libturbo_b200_selfcheck.so")


def build_selfcheck(force=False):
    """Test-only device checks (csrc/test/*.cu) in a library of their own, so
    that nothing the product library exports exists only for the tests."""
    srcs = sorted(glob.glob(os.path.join(SELFCHECK_SRCS, "*.cu")))
    newest = max(os.path.getmtime(f) for f in srcs + headers())
    if not force and os.path.exists(SELFCHECK_OUT) and os.path.getmtime(SELFCHECK_OUT) >= newest:
        return SELFCHECK_OUT
    cmd = [NVCC] + FLAGS + ["-shared", "-o", SELFCHECK_OUT] + srcs
    subprocess.check_call(cmd)
    return SELFCHECK_OUT


HOST = os.path.join(HERE, "host")
HOST_OUT = os.path.join(HERE, "libturbo_b200_host.so")
CXX = os.environ.get("CXX_HOST", "/usr/bin/g++")


def build_host(force=False):
    """The C++ Tensor/nn/MiniGPT layer over the C ABI (no CUDA headers)."""
    srcs = sorted(glob.glob(os.path.join(HOST, "src", "*.cpp")))
    hdrs = glob.glob(os.path.join(HOST, "src", "*.hpp")) + glob.glob(os.path.join(HOST, "include", "turbo", "*", "*.hpp"))
    test_src = os.path.join(HOST, "tests", "test_host.cpp")
    test_bin = os.path.join(HOST, "tests", "test_host")
    newest = max(os.path.getmtime(f) for f in srcs + hdrs + [OUT, test_src])
    if (not force and os.path.exists(HOST_OUT) and os.path.exists(test_bin)
            and min(os.path.getmtime(HOST_OUT), os.path.getmtime(test_bin)) >= newest):
        return HOST_OUT
    cmd = [CXX, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wno-reorder",
           "-I" + os.path.join(HOST, "include"), "-I" + os.path.join(ROOT, "include")] + srcs + \
          ["-L" + HERE, "-lturbo_b200", "-Wl,-rpath,$ORIGIN", "-o", HOST_OUT]
    subprocess.check_call(cmd)
    # the C++ test program (reference unit-test cases against this API)
    test_src = os.path.join(HOST, "tests", "test_host.cpp")
    cmd = [CXX, "-std=c++17", "-O2", "-Wall", "-I" + os.path.join(HOST, "include"), test_src,
           "-L" + HERE, "-lturbo_b200_host", "-lturbo_b200", "-Wl,-rpath,$ORIGIN/../..",
           "-o", os.path.join(HOST, "tests", "test_host")]
    subprocess.check_call(cmd)
    return HOST_OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
