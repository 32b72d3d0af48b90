"""Build the package's native code in-tree (no GPU needed; nvcc cross-compiles for sm_100a).

Outputs, next to this file:
  libnvfp4_b200.so                 CUDA kernels + the C ABI of include/nvfp4_b200.h
  my_plugins<EXT_SUFFIX>           the torch/pybind11 module (linked to libnvfp4_b200.so)

Usage:  python -m my_nvfp4_gemm_b200.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", f"-I{INCLUDE}"] + ARCH

CU_SOURCES = ["quantize.cu", "gemm_sm100.cu", "scale_layout.cu", "peer.cu"]
HEADERS = ["ptx.cuh", "capi_util.h", "block_quant.cuh"]

LIB_NAME = "libnvfp4_b200.so"
EXT_NAME = "my_plugins"


def lib_path() -> str:
    return os.path.join(HERE, LIB_NAME)


def ext_path() -> str:
    return os.path.join(HERE, EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_lib(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "nvfp4_b200.h")]
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        list(ex.map(_run, jobs))
    out = lib_path()
    exports = os.path.join(CSRC, "exports.map")
    if force or jobs or _newer(out, objs + [exports]):
        _run([NVCC, "-shared"] + ARCH + ["-Xlinker", f"--version-script={exports}", "-o", out] + objs)
    return out


def build_ext(force: bool = False) -> str:
    import torch  # noqa: F401  (build-time only: include/library paths and ABI flag)
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_binding.cpp")
    out = ext_path()
    if not (force or _newer(out, [src, os.path.join(INCLUDE, "nvfp4_b200.h"), lib_path()])):
        return out
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")]
    incs.append(f"-I{sysconfig.get_paths()['include']}")
    libdirs = [f"-L{p}" for p in ce.library_paths(device_type="cuda")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = (["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wno-unused-function",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
            "-DTORCH_API_INCLUDE_EXTENSION_H", f"-I{INCLUDE}", src, "-o", out]
           + incs + libdirs
           + ["-L" + HERE, "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN",
              "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-ltorch_cuda"])
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(lib_path())
    print(ext_path())
