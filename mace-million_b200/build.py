#!/usr/bin/env python
"""Build libmace_b200.so (all CUDA sources of csrc/, sm_100a) in-tree: mace_onegpu/_lib/libmace_b200.so.

    python mace-million_b200/build.py [--force]

Plain nvcc, no torch extension machinery: the library exposes a C ABI (include/mace_b200.h) and is loaded with
ctypes.  Rebuilds only when a source is newer than the library (or with --force).
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "mace_onegpu", "_lib", "libmace_b200.so")
INC = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-O3", "--expt-relaxed-constexpr", f"-I{INC}"]


OPS_SRC = os.path.join(CSRC, "torch_ops.cpp")
OPS_OUT = os.path.join(HERE, "mace_onegpu", "_lib", "libmace_b200_torch.so")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INC, "mace_b200.h")]


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(p) > t for p in deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [NVCC, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(out.decode())
            raise RuntimeError(f"nvcc failed on {src}")
    tmp = OUT + ".tmp"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp, "-lcudart"]
    subprocess.check_call(cmd)
    os.replace(tmp, OUT)
    return OUT


def build_ops(force: bool = False, verbose: bool = False) -> str:
    """libmace_b200_torch.so: the TORCH_LIBRARY(mace_b200) custom ops (csrc/torch_ops.cpp), host C++ compiled against
    torch's headers and linked to libmace_b200.so (loaded with torch.ops.load_library)."""
    lib = build(force, verbose)
    if not force and os.path.exists(OPS_OUT) and all(os.path.getmtime(p) <= os.path.getmtime(OPS_OUT)
                                                     for p in (OPS_SRC, lib, os.path.join(INC, "mace_b200.h"))):
        return OPS_OUT
    import torch

    cuda_home = os.path.dirname(os.path.dirname(NVCC))
    tdir = os.path.dirname(torch.__file__)
    inc = [os.path.join(tdir, "include"), os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
           os.path.join(cuda_home, "include"), INC]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    # the system g++ (the one torch's own extensions use): a C++ exception thrown by an op (TORCH_CHECK) has to unwind
    # through libtorch, and objects linked by a compiler driver with its own support-library directories crashed there
    cxx = os.environ.get("MACE_B200_CXX") or ("/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
    tmp = OPS_OUT + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in inc], OPS_SRC, "-o", tmp,
           f"-L{os.path.join(tdir, 'lib')}", f"-L{os.path.dirname(lib)}", f"-L{os.path.join(cuda_home, 'lib64')}",
           "-lmace_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{os.path.join(tdir, 'lib')}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(tmp, OPS_OUT)
    return OPS_OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_ops(force="--force" in sys.argv, verbose=True))
