"""Builds libmcb200.so, the sm_100a C-ABI library of the KV-cache decode path, in-tree.

    python -m modelcore_b200.build            # compile if a source is newer than the library
    python -m modelcore_b200.build --force    # always recompile

The library is a single translation unit (csrc/mcb200.cu) compiled by nvcc for sm_100a only,
with the CUDA runtime linked statically so that loading it needs no CUDA driver (the CPU test
suite checks the exported symbols without a GPU).
"""
import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
REPO = os.path.dirname(PKG_DIR)
INCLUDE = os.path.join(REPO, "include")
LIB_PATH = os.path.join(PKG_DIR, "libmcb200.so")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    out = []
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                out.append(os.path.join(d, name))
    return out


def _nvcc():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmcb200.so")
    return nvcc


def needs_build(lib_path=LIB_PATH):
    if not os.path.exists(lib_path):
        return True
    t = os.path.getmtime(lib_path)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force=False, verbose=False, lib_path=LIB_PATH):
    """Compiles csrc/mcb200.cu into lib_path (default: modelcore_b200/libmcb200.so)."""
    if not force and not needs_build(lib_path):
        return lib_path
    tmp = lib_path + ".tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "--cudart", "static",
           "-Xcompiler", "-fPIC", "-shared", "-I", INCLUDE, "-o", tmp,
           os.path.join(CSRC, "mcb200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, lib_path)
    return lib_path


TORCH_OPS_PATH = os.path.join(PKG_DIR, "libmcb200_torch.so")
TORCH_OPS_SRC = os.path.join(CSRC, "torch_ops.cpp")


def torch_ops_needs_build(path=TORCH_OPS_PATH):
    if not os.path.exists(path):
        return True
    t = os.path.getmtime(path)
    deps = (TORCH_OPS_SRC, os.path.join(INCLUDE, "mcb200.h"), LIB_PATH)
    return any(os.path.getmtime(s) > t for s in deps)


def _torch_paths():
    import torch.utils.cpp_extension as ce
    try:
        incs = ce.include_paths(device_type="cuda")
    except TypeError:
        incs = ce.include_paths(cuda=True)
    import torch
    return incs, os.path.join(os.path.dirname(torch.__file__), "lib")


def build_torch_ops(force=False, path=TORCH_OPS_PATH):
    """Compiles csrc/torch_ops.cpp -- the torch.ops.mcb200 operators over the C ABI -- against the
    installed torch into path (default: modelcore_b200/libmcb200_torch.so), linked to
    libmcb200.so beside it (built first when missing or stale)."""
    build()
    if not force and not torch_ops_needs_build(path):
        return path
    import torch
    incs, torch_lib = _torch_paths()
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler found to build libmcb200_torch.so")
    tmp = path + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    for inc in incs:
        cmd += ["-isystem", inc]
    cmd += [TORCH_OPS_SRC, "-o", tmp, "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-L", PKG_DIR, "-lmcb200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("c++ failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    os.replace(tmp, path)
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill usage")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    print(build_torch_ops(force=args.force))


if __name__ == "__main__":
    main()
