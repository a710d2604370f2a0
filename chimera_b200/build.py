"""Build recipe for the native parts of chimera_b200 (in-tree, no JIT cache).

* ``lib/libchimera_b200.so`` -- the CUDA kernels and the C ABI
  (include/chimera_b200.h), compiled for sm_100a only.
* ``lib/libchimera_nccl.so`` -- the document-sharded search over NCCL
  (include/chimera_b200_sharded.h).
* ``lib/libchimera_core.so`` -- the drop-in C++ ``Chimera::chimera_index``
  (include/chimera/chimera_index.cuh) over the C ABI.
* ``chimera*.so`` (this directory) -- the pybind11 module ``chimera``.
* ``bin/gpu_build``, ``bin/gpu_search`` -- the drop-in CLI tools.

Run ``python -m chimera_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
BIN = os.path.join(HERE, "bin")
OBJ = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE,
                     "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]

CU_SOURCES = ["capi.cu", "query_prep.cu", "probe.cu", "stage1.cu", "refine.cu", "build.cu", "tcgemm.cu",
              "shard.cu", "refine_tc.cu", "stage1_bound.cu"]
HOST_SOURCES = ["host/chimera_index.cpp", "host/io.cpp", "host/rng.cpp"]


def _cxx():
    # the image may export CC/CXX wrappers that lack libgomp; use the system g++
    return shutil.which("g++") or "g++"


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    out = []
    for d in (CSRC, os.path.join(CSRC, "host"), os.path.join(CSRC, "apps"), INCLUDE,
              os.path.join(INCLUDE, "chimera")):
        if os.path.isdir(d):
            out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh", ".hpp"))]
    return out


def build_cuda(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    hdrs = _headers()
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace("/", "_") + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for log in ex.map(_run, jobs):
            if verbose and log.strip():
                print(log)
    so = os.path.join(LIB, "libchimera_b200.so")
    if _stale(so, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", so] + objs + ["-lcudart"])  # driver API via entry points
    # the document-sharded search over NCCL: its own library, so that the core
    # one has no NCCL dependency
    src = os.path.join(CSRC, "sharded.cu")
    obj = os.path.join(OBJ, "sharded.cu.o")
    if _stale(obj, [src] + hdrs):
        _run([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    nso = os.path.join(LIB, "libchimera_nccl.so")
    if _stale(nso, [obj, so]):
        _run([NVCC] + ARCH + ["-shared", "-o", nso, obj, "-L" + LIB, "-lchimera_b200", "-lnccl", "-lcudart",
                              "-Xlinker", "-rpath,$ORIGIN"])
    return so


def build_host(verbose=False):
    os.makedirs(LIB, exist_ok=True)
    os.makedirs(BIN, exist_ok=True)
    cxx = _cxx()
    inc = ["-I" + INCLUDE, "-I" + os.path.join(CUDA_HOME, "include")]
    cflags = ["-std=c++17", "-O2", "-fPIC"] + inc
    hdrs = _headers()
    core = os.path.join(LIB, "libchimera_core.so")
    srcs = [os.path.join(CSRC, s) for s in HOST_SOURCES]
    rpath = "-Wl,-rpath,$ORIGIN"
    if _stale(core, srcs + hdrs + [os.path.join(LIB, "libchimera_b200.so")]):
        _run([cxx] + cflags + ["-shared", "-o", core] + srcs +
             ["-L" + LIB, "-lchimera_b200", "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart", rpath])
    # CLI tools
    for tool in ("gpu_build", "gpu_search"):
        exe = os.path.join(BIN, tool)
        srcs_t = [os.path.join(CSRC, "apps", tool + ".cpp"), os.path.join(CSRC, "apps", "cli.cpp")]
        if _stale(exe, srcs_t + hdrs + [core]):
            _run([cxx] + cflags + ["-I" + os.path.join(CSRC, "apps"), "-o", exe] + srcs_t +
                 ["-L" + LIB, "-lchimera_core", "-lchimera_b200", "-L" + os.path.join(CUDA_HOME, "lib64"),
                  "-lcudart", "-Wl,-rpath,$ORIGIN/../lib"])
    # pybind11 module `chimera`
    import pybind11
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    mod = os.path.join(HERE, "chimera" + ext)
    psrc = os.path.join(CSRC, "python", "bindings.cpp")
    if _stale(mod, [psrc, core] + hdrs):
        _run([cxx] + cflags + ["-shared", "-o", mod, psrc, "-I" + pybind11.get_include(),
                               "-I" + sysconfig.get_paths()["include"], "-L" + LIB, "-lchimera_core",
                               "-lchimera_b200", "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart",
                               "-Wl,-rpath,$ORIGIN/lib"])
    return core


def build_hostrng():
    os.makedirs(LIB, exist_ok=True)
    so = os.path.join(LIB, "libchimera_hostrng.so")
    src = os.path.join(CSRC, "host", "rng.cpp")
    if _stale(so, [src]):
        _run([_cxx(), "-std=c++17", "-O2", "-fPIC", "-shared", "-o", so, src])
    return so


def build(verbose=False, host=True):
    build_cuda(verbose)
    build_hostrng()
    if host:
        build_host(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", LIB)
