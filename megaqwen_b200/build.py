"""Build the native parts in-tree (no JIT cache, so the built files travel with
the source tree to GPU hosts).

Outputs
-------
``megaqwen_b200/lib/libmegaqwen_b200.so``  the C-ABI library (CUDA kernels for
    sm_100a + extern "C" entry points in ``include/megaqwen_b200.h``); links the
    CUDA runtime statically and has no torch dependency.
``megaqwen_b200/_C<ext-suffix>``           the torch extension exposing the
    reference's classes, linked against the library above.

Run ``python megaqwen_b200/build.py`` (or ``__graft_entry__.build()``).  Each
output is rebuilt only when a source it depends on is newer.
``MQ_DECODE_TRACE=1 python megaqwen_b200/build.py --force`` builds the decode
kernel with its per-phase/per-tile trace stamps (``mq_decode_params.trace``);
the default build leaves them out.  ``MQ_PROFILE_HOOKS=1`` likewise compiles
the batched-decode and prefill profiling hooks (off by default).
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmegaqwen_b200.so"
EXT = PKG / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["decode.cu", "prefill.cu", "decode_batch.cu"]
CUDA_HEADERS = ["mq_ptx.cuh", "mq_tc.cuh", "gemm_tc.cuh", "gemm_small.cuh", "gemm_persist.cuh", "gemm_pair.cuh", "attn_tc.cuh", "prefill_kernels.cuh", "attn_fa.cuh"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(home) / "bin" / "nvcc")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {r.returncode})")
    return r.stdout + r.stderr


def build_lib(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in CUDA_SOURCES]
    deps = srcs + [CSRC / h for h in CUDA_HEADERS] + [INCLUDE / "megaqwen_b200.h", Path(__file__)]
    if not force and not _stale(LIB, deps):
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    cmd = [_nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}", *srcs, "-o", LIB]
    if os.environ.get("MQ_DECODE_TRACE") == "1":
        cmd.insert(1, "-DMQ_DECODE_TRACE=1")
    if os.environ.get("MQ_PROFILE_HOOKS") == "1":
        cmd.insert(1, "-DMQ_PROFILE_HOOKS=1")
    out = _run(cmd, verbose)
    (LIBDIR / "ptxas_info.txt").write_text(out)
    return LIB


def build_ext(verbose: bool = False, force: bool = False) -> Path:
    import torch
    import torch.utils.cpp_extension as ce
    import pybind11

    src = CSRC / "ext.cpp"
    deps = [src, INCLUDE / "megaqwen_b200.h", LIB, Path(__file__)]
    if not force and not _stale(EXT, deps):
        return EXT
    incs = ce.include_paths(device_type="cuda") + [pybind11.get_include(), sysconfig.get_paths()["include"],
                                                    str(INCLUDE)]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", "-w",
           *[f"-I{i}" for i in incs], str(src), "-o", str(EXT),
           *[f"-L{d}" for d in libdirs if "torch" in d], f"-L{LIBDIR}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lmegaqwen_b200",
           "-Wl,-rpath,$ORIGIN/lib"]
    _run(cmd, verbose)
    return EXT


def build(verbose: bool = False, force: bool = False):
    lib = build_lib(verbose, force)
    ext = build_ext(verbose, force)
    return lib, ext


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    print("built", LIB, EXT)
