"""Build the in-tree native artefacts of tecoops-b200.

    python teco-ops_b200/build.py            # everything
    python teco-ops_b200/build.py --jobs 8

Products (all written next to the sources, so they travel with the repository
snapshot; object files go to teco-ops_b200/_build/):
  teco-ops_b200/tecoops/libteco_ops.so         C-ABI library (include/tecoops.h):
                                               interface + UAL + sm_100a kernels
  teco-ops_b200/tecoops/_torch_ext*.so         PyTorch binding (pybind `_torch_ext`
                                               + TORCH_LIBRARY(tecoops))
  teco-ops_b200/tecoops/libteco_ops_plugin.so  inference plugins, compiled against
                                               the stand-in plugin SDK header
  oracle/liboracle_rc.so                       CPU restatement of the reshape golden
                                               (test infrastructure)

Every CUDA translation unit is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a).  Rebuilds are incremental on file
modification times (headers included).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
OUT = os.path.join(PKG, "tecoops")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_INC = "/usr/local/cuda/include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCS = ["-I" + CSRC, "-I" + os.path.join(ROOT, "include")]

LIB = os.path.join(OUT, "libteco_ops.so")
PLUGIN = os.path.join(OUT, "libteco_ops_plugin.so")
ORACLE = os.path.join(ROOT, "oracle", "liboracle_rc.so")


def _headers():
    hs = []
    for pat in ("**/*.h", "**/*.hpp", "**/*.cuh"):
        hs += glob.glob(os.path.join(CSRC, pat), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def _lib_sources():
    srcs = []
    for sub in ("interface", "ual"):
        for ext in ("*.cu", "*.cpp"):
            srcs += glob.glob(os.path.join(CSRC, sub, "**", ext), recursive=True)
    return sorted(srcs)


def build_lib(jobs: int, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = _headers()
    objs, work = [], []
    for src in _lib_sources():
        rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
        obj = os.path.join(BUILD, rel + ".o")
        objs.append(obj)
        if _stale(obj, [src] + hdrs):
            if src.endswith(".cu"):
                cmd = [NVCC, *ARCH, "-lineinfo", "-std=c++17", "-O3", "-Xcompiler", "-fPIC",
                       *INCS, "-c", src, "-o", obj]
                if verbose:
                    cmd += ["-Xptxas", "-v"]
            else:
                cmd = ["g++", "-std=c++17", "-O2", "-fPIC", *INCS, "-I" + CUDA_INC, "-c", src,
                       "-o", obj]
            work.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(_run, work):
            if verbose and out:
                print(out)
    if _stale(LIB, objs):
        _run([NVCC, "-shared", *ARCH, "-o", LIB, *objs, "-Xlinker", "--no-undefined",
              "-lcudart_static", "-ldl", "-lrt", "-lpthread"])
    return LIB


def build_oracle() -> str:
    src = os.path.join(ROOT, "oracle", "reshape_and_cache.c")
    if _stale(ORACLE, [src]):
        _run(["gcc", "-O2", "-shared", "-fPIC", "-o", ORACLE, src, "-lpthread"])
    return ORACLE


def build_plugin() -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "plugin", "**", "*.cc"), recursive=True))
    cus = sorted(glob.glob(os.path.join(CSRC, "plugin", "**", "*.cu"), recursive=True))
    if not srcs:
        return ""
    pinc = "-I" + os.path.join(CSRC, "plugin")
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for cu in cus:   # the plugins' own small kernels (sm_100a)
        obj = os.path.join(BUILD, "plugin_" + os.path.basename(cu) + ".o")
        objs.append(obj)
        if _stale(obj, [cu] + _headers()):
            _run([NVCC, *ARCH, "-lineinfo", "-std=c++17", "-O3", "-Xcompiler", "-fPIC", *INCS,
                  pinc, "-c", cu, "-o", obj])
    deps = srcs + objs + _headers() + [LIB]
    if _stale(PLUGIN, deps):
        _run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", *INCS, pinc, "-I" + CUDA_INC,
              "-o", PLUGIN, *srcs, *objs, "-L" + OUT, "-lteco_ops", "-L/usr/local/cuda/lib64",
              "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-Wl,-rpath,$ORIGIN",
              "-Wl,--no-undefined"])
    return PLUGIN


def torch_ext_path() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(OUT, "_torch_ext" + suffix)


def build_torch_ext() -> str:
    src = os.path.join(CSRC, "api", "torch_ext.cpp")
    if not os.path.exists(src):
        return ""
    target = torch_ext_path()
    if not _stale(target, [src] + _headers() + [LIB]):
        return target
    import torch
    from torch.utils import cpp_extension as ce
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = ["-I" + p for p in ce.include_paths(device_type="cuda")]
    incs += ["-I" + sysconfig.get_paths()["include"], "-I" + CUDA_INC]
    libdirs = ["-L" + p for p in ce.library_paths(device_type="cuda")]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    _run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          "-DTORCH_EXTENSION_NAME=_torch_ext", "-DTORCH_API_INCLUDE_EXTENSION_H", *INCS, *incs,
          src, "-o", target, *libdirs, "-L" + OUT, "-lteco_ops", "-lc10", "-lc10_cuda",
          "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
          "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + torch_lib])
    return target


def build_all(jobs: int = 8, verbose: bool = False, torch_ext: bool = True) -> dict:
    out = {"lib": build_lib(jobs, verbose), "oracle": build_oracle()}
    out["plugin"] = build_plugin()
    if torch_ext:
        out["torch_ext"] = build_torch_ext()
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--no-torch", action="store_true")
    a = ap.parse_args()
    res = build_all(a.jobs, a.verbose, not a.no_torch)
    for k, v in res.items():
        print(f"{k}: {v}")
    sys.exit(0)
