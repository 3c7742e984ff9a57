"""In-tree build of the native libraries (no JIT cache, no setuptools).

* ``libgdn_rssm_b200.so`` -- the CUDA kernels and the C ABI declared in
  ``include/gdn_recoverssm_b200.h`` (nvcc, ``-gencode arch=compute_100a,
  code=sm_100a``; cudart linked statically, so the library has no torch
  dependency).
* ``_C.so`` -- the torch custom ops (``torch.ops.gdn_recoverssm_ac.*``) over
  that C ABI (g++ against the installed torch headers).

Both land next to this file so that they travel with the source tree.  A
rebuild happens only when a source or header is newer than the output.

    python -m gdn_recoverssm_b200.build [--force] [--jobs N]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent.parent / "include"
OBJ = PKG / "_build"
CAPI_LIB = PKG / "libgdn_rssm_b200.so"
TORCH_LIB = PKG / "_C.so"

CUDA_SOURCES = ["capi.cu", "fold.cu", "verify_bf16.cu", "verify_f16.cu", "verify_f32.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("GDN RecoverSSM build: nvcc not found (set CUDA_HOME)")


def _host_cxx() -> str:
    """The C++ compiler of the torch-op library: ``GDN_RSSM_CXX``, else the
    ``g++`` on PATH.  The library must link the SHARED C++ runtime that torch
    itself uses: a private static copy (what a toolchain whose shared
    libstdc++ link is missing produces) gives the library its own iostreams
    and exception runtime, and formatting a TORCH_CHECK message there crashes
    the process.  ``_check_shared_runtime`` refuses such a build."""
    return os.environ.get("GDN_RSSM_CXX") or shutil.which("g++") or os.environ.get("CXX", "g++")


def _check_shared_runtime(lib: Path) -> None:
    nm = shutil.which("nm")
    if nm is None:
        return
    out = subprocess.run([nm, "-D", "--defined-only", str(lib)], capture_output=True, text=True).stdout
    if "__cxa_throw" in out or "_ZNSt8ios_base4InitC" in out:
        lib.unlink()
        raise RuntimeError(
            f"GDN RecoverSSM build: {lib.name} embeds a static C++ runtime (its compiler linked libstdc++.a); "
            "build it with a g++ that links the shared libstdc++ (set GDN_RSSM_CXX)"
        )


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(output: Path, inputs) -> bool:
    if not output.exists():
        return True
    t = output.stat().st_mtime
    return any(Path(i).stat().st_mtime > t for i in inputs)


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "GDN RecoverSSM build failed:\n  " + " ".join(map(str, cmd)) + "\n" + proc.stdout + proc.stderr
        )
    return proc


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> dict:
    """Build both libraries if stale; returns their paths."""
    cuda = _cuda_home()
    nvcc = str(cuda / "bin" / "nvcc")
    OBJ.mkdir(exist_ok=True)
    headers = _headers()
    flags = [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
    ]

    def compile_one(name):
        src = CSRC / name
        obj = OBJ / (name + ".o")
        if force or _stale(obj, [src, *headers]):
            _run([nvcc, *flags, "-c", str(src), "-o", str(obj)])
            if verbose:
                print("compiled", name, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, CUDA_SOURCES))
    if force or _stale(CAPI_LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-o", str(CAPI_LIB), *map(str, objs)])
        _check_shared_runtime(CAPI_LIB)
        if verbose:
            print("linked", CAPI_LIB.name, flush=True)

    src = CSRC / "torch_ops.cpp"
    if force or _stale(TORCH_LIB, [src, CAPI_LIB, *headers]):
        import torch
        from torch.utils import cpp_extension

        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        incs = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{cuda / 'include'}", f"-I{INCLUDE}"]
        libdirs = cpp_extension.library_paths()
        cmd = [
            _host_cxx(),
            "-O2",
            "-std=c++17",
            "-fPIC",
            "-shared",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
            *incs,
            str(src),
            "-o",
            str(TORCH_LIB),
            *[f"-L{d}" for d in libdirs],
            f"-L{PKG}",
            "-lgdn_rssm_b200",
            "-lc10",
            "-lc10_cuda",
            "-ltorch_cpu",
            "-ltorch",
            "-Wl,-rpath,$ORIGIN",
            *[f"-Wl,-rpath,{d}" for d in libdirs],
        ]
        _run(cmd)
        _check_shared_runtime(TORCH_LIB)
        if verbose:
            print("linked", TORCH_LIB.name, flush=True)
    return {"capi": CAPI_LIB, "torch": TORCH_LIB}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    out = build(force=args.force, jobs=args.jobs, verbose=True)
    for k, v in out.items():
        print(k, v)


if __name__ == "__main__":
    sys.exit(main())
