"""Build recipe for the checkers under oracle/ (test infrastructure only).

* ``oracle/liboracle.so`` -- the C restatement in ``gemm_oracle.c`` (gcc,
  pthreads, x86-64-v3 so it runs on any recent server CPU).
* ``oracle/_ref/libref_gemm.so`` -- the reference's own GEMM kernels, compiled
  with nvcc from their sources where they lie in the reference checkout
  (``src/kernels/kernel_v1.cu`` ... ``kernel_v8.cu``; nothing is copied), with
  the flags the reference's harness uses (``-O3 -lineinfo
  -gencode=arch=compute_100a,code=sm_100a``, ``-lcuda``;
  src/bench_core.py:36-43), plus ``ref_shim.cu`` for a C entry point.  The
  kernel files include torch headers and use TORCH_CHECK, so torch's include
  directories and libc10 are on the command line.  This step runs only where
  the reference checkout exists (``B200_REFERENCE_DIR``, by default a
  directory named ``reference`` beside this repository); the built library is
  what travels to the GPU machine.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_SO = REF_DIR / "libref_gemm.so"
# The reference checkout: B200_REFERENCE_DIR, else a checkout named
# "reference" beside this repository's directory.
REFERENCE_DIR = Path(os.environ.get("B200_REFERENCE_DIR", HERE.parent.parent / "reference"))
REF_VERSIONS = ["v1", "v2", "v3", "v4", "v5", "v6", "v7", "v8"]


def _run(cmd, verbose=False):
    if verbose:
        print(" ".join(map(str, cmd)), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stale(out: Path, inputs) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(i).stat().st_mtime > t for i in inputs)


def build_oracle(force=False, verbose=False) -> Path:
    src = HERE / "gemm_oracle.c"
    if force or _stale(ORACLE_SO, [src]):
        tmp = ORACLE_SO.with_suffix(".tmp")
        _run(["gcc", "-O3", "-march=x86-64-v3", "-fPIC", "-shared", "-pthread", "-std=c11",
              src, "-o", tmp], verbose)
        os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def reference_sources():
    kdir = REFERENCE_DIR / "src" / "kernels"
    return [kdir / f"kernel_{v}.cu" for v in REF_VERSIONS]


def build_ref(force=False, verbose=False):
    """Compile the reference kernels; returns the .so path or None if the
    reference checkout is absent (the prebuilt library is then used as is)."""
    srcs = reference_sources()
    if not all(s.exists() for s in srcs):
        return REF_SO if REF_SO.exists() else None
    shim = HERE / "ref_shim.cu"
    if not force and not _stale(REF_SO, srcs + [shim, REFERENCE_DIR / "src" / "profiler.h"]):
        return REF_SO
    import torch
    import torch.utils.cpp_extension as cpp

    REF_DIR.mkdir(exist_ok=True)
    obj_dir = REF_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    common = [nvcc, "-std=c++17", "-O3", "-lineinfo", "-gencode=arch=compute_100a,code=sm_100a",
              "-Xcompiler", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              *[f"-I{p}" for p in cpp.include_paths()]]

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        _run(common + ["-c", src, "-o", obj], verbose)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs + [shim]))
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    tmp = REF_SO.with_suffix(".tmp")
    _run([nvcc, "-shared", *objs, "-o", tmp, f"-L{torch_lib}", "-lc10",
          f"-L{cuda_home}/lib64/stubs", "-lcuda", f"-Xlinker", f"-rpath,{torch_lib}"], verbose)
    os.replace(tmp, REF_SO)
    shutil.rmtree(obj_dir, ignore_errors=True)
    return REF_SO


def build(force=False, verbose=False):
    build_oracle(force, verbose)
    build_ref(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print("oracle built:", ORACLE_SO, REF_SO if REF_SO.exists() else "(no reference)")
