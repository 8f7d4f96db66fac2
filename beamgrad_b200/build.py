# SPDX-License-Identifier: MIT
"""In-tree build of the engine's native libraries.

* ``beamgrad_b200/libdbs_cuda.so`` -- the C ABI of include/dbs_cuda.h (+ dbs_cuda_b200.h),
  CUDA kernels for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), built with
  ``-fmad=false`` and IEEE division so no multiply-add is ever contracted.
* ``beamgrad_b200/_C_cuda*.so`` -- the torch operator module (``torch.ops.beamgrad.*`` CUDA
  kernels), a thin C++ layer over the C ABI.

Run ``python -m beamgrad_b200.build`` (or call :func:`build`). nvcc cross-compiles without
a GPU. Outputs stay in the package directory so they travel with the repository snapshot.
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
LIB = PKG / "libdbs_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-fmad=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-ffp-contract=off,-fvisibility=hidden",
]
LIB_SOURCES = ["decode.cu", "decode_f32.cu", "decode_f16.cu", "decode_bf16.cu", "backward.cu", "api.cu", "static_scratch.cu",
               "vshard.cu", "search.cu", "pool.cu"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}):\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    deps = [CSRC / s for s in LIB_SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    from concurrent.futures import ThreadPoolExecutor

    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))

    def compile_one(src: str) -> tuple[str, str]:
        obj = build_dir / (Path(src).stem + ".o")
        if not force and not ptxas_info and not _stale(obj, [CSRC / src, *headers]):
            return str(obj), ""
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        return str(obj), _run(cmd, verbose)

    with ThreadPoolExecutor(max_workers=min(len(LIB_SOURCES), os.cpu_count() or 4)) as pool:
        results = list(pool.map(compile_one, LIB_SOURCES))
    objs = [obj for obj, _ in results]
    if ptxas_info:
        for _, out in results:
            print(out)
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH, "-shared", "-Xlinker", "-soname,libdbs_cuda.so.10", "-o", str(tmp), *objs, "-lcudart"], verbose)
    os.replace(tmp, LIB)
    soname = PKG / "libdbs_cuda.so.10"  # what modules linked against the library ask for
    if soname.is_symlink() or soname.exists():
        soname.unlink()
    soname.symlink_to(LIB.name)
    return LIB


def torch_ext_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / f"_C_cuda{suffix}"


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """The torch operator module, compiled with g++ against torch's headers; links libdbs_cuda.so."""
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    out = torch_ext_path()
    if not src.exists():
        return out
    if not force and not _stale(out, [src, LIB, *INCLUDE.glob("*.h")]):
        return out
    includes = cpp_extension.include_paths(device_type="cuda") if "device_type" in cpp_extension.include_paths.__code__.co_varnames else cpp_extension.include_paths(cuda=True)
    # The module must share torch's C++ runtime: errors raised in an operator are C++
    # exceptions caught inside torch, which breaks if libstdc++ is linked statically
    # (as some compiler wrappers do). Use the system compiler and verify below.
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else os.environ.get("CXX", "g++")
    py_inc = sysconfig.get_paths()["include"]
    torch_lib = Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C_cuda", "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{p}" for p in includes], f"-I{py_inc}", f"-I{INCLUDE}", "-I/usr/local/cuda/include",
        str(src), "-o", str(out.with_suffix(".tmp")),
        f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
        f"-L{PKG}", "-l:libdbs_cuda.so", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
        "-L/usr/local/cuda/lib64", "-lcudart",
    ]
    _run(cmd, verbose)
    syms = subprocess.run(["nm", "-D", "--defined-only", str(out.with_suffix(".tmp"))], capture_output=True, text=True).stdout
    if " __cxa_throw" in syms:
        raise RuntimeError(f"{out.name} carries its own copy of libstdc++ (built by {cxx}); torch could not catch its errors")
    os.replace(out.with_suffix(".tmp"), out)
    return out


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_torch_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    force = "--force" in sys.argv
    build_lib(force=force, verbose=True, ptxas_info="--ptxas" in sys.argv)
    if "--no-torch" not in sys.argv:
        build_torch_ext(force=force, verbose=True)
