"""In-tree build of the native parts of blackwell_gemm_b200.

Two artefacts, both written next to this file so they travel with the source
tree and are found without installation:

* ``libb200gemm.so`` -- the sm_100a kernels and the C ABI of
  ``include/b200_gemm.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static CUDA runtime, the driver's tensor-map encoder looked up at run time so
  no ``-lcuda`` is needed);
* ``_C<ext-suffix>`` -- the torch extension with the reference-compatible
  ``matmul_b200`` / ``profile_matmul_b200`` entry points, linked against
  ``libb200gemm.so`` through ``$ORIGIN``.

Each step is skipped when its output is newer than all of its inputs.
Run ``python -m blackwell_gemm_b200.build`` to build by hand.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libb200gemm.so"
EXT = PKG / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = shutil.which("nvcc") or os.path.join(cuda_home, "bin", "nvcc")
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")
    return cand


def _stale(out: Path, inputs) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(i).stat().st_mtime > t for i in inputs)


def _run(cmd, verbose: bool) -> str:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}):\n{' '.join(map(str, cmd))}\n"
                           f"{res.stdout}\n{res.stderr}")
    return res.stdout + res.stderr


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    srcs = [CSRC / "gemm_capi.cu", CSRC / "gemm_kernel.cuh", CSRC / "gemm_layout.h",
            CSRC / "gemm_skinny.cuh", CSRC / "ksplit_fused.cuh", CSRC / "sm100_ptx.cuh",
            INCLUDE / "b200_gemm.h"]
    if not force and not _stale(LIB, srcs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    log = _run([_nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS, "-Xptxas", "-v",
                "-I", INCLUDE, "-I", CSRC, "-shared", "-Xcompiler", "-fPIC",
                "-o", tmp, CSRC / "gemm_capi.cu"], verbose)
    os.replace(tmp, LIB)
    (PKG / "_build_ptxas.txt").write_text(log)
    return LIB


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    srcs = [CSRC / "matmul.cpp", INCLUDE / "b200_gemm.h", LIB]
    if not force and not _stale(EXT, srcs):
        return EXT
    import torch
    import torch.utils.cpp_extension as cpp

    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = cpp.include_paths() + [os.path.join(cuda_home, "include"),
                                  sysconfig.get_paths()["include"], str(INCLUDE)]
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    tmp = EXT.with_suffix(".tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H", *[f"-I{i}" for i in incs],
           CSRC / "matmul.cpp", "-o", tmp,
           f"-L{PKG}", "-lb200gemm", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd, verbose)
    os.replace(tmp, EXT)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force, verbose)
    build_ext(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(f"built {LIB.name} and {EXT.name}")
