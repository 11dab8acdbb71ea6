"""Build recipe for the reference decode megakernel on sm_100a (comparator).

TEST AND BENCHMARK INFRASTRUCTURE ONLY.  Compiles the reference's own
``csrc/megakernel/fused_decode_ldg.cu`` (the cooperative 82 x 256 grid.sync
kernel plus its two LM-head kernels and the ``launch_ldg_decode`` /
``launch_ldg_decode_with_logits`` launchers) unchanged, from where it lies in
the reference tree, with ``-gencode arch=compute_100a,code=sm_100a`` in place
of the ``-arch=sm_86`` of ``megakernel_decode.py:255``.  The output goes to
``oracle/_ref/libref_ldg_decode.so`` (git-ignored; it travels to GPU hosts with
the working tree).  No reference source is copied into this repository.

``bench.py`` times it next to this engine (``reference_megakernel_sm100a``);
the product never loads it.

Run: ``python oracle/build_ref.py [REFERENCE_ROOT]`` (default: the
``MEGAQWEN_REFERENCE`` environment variable).  Without a reference tree the
build is skipped and an existing library is kept.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libref_ldg_decode.so"
SOURCE = Path("csrc") / "megakernel" / "fused_decode_ldg.cu"   # relative to the reference root


def build(reference_root: str | None = None, verbose: bool = False) -> Path | None:
    root = reference_root or os.environ.get("MEGAQWEN_REFERENCE")
    if not root or not (Path(root) / SOURCE).exists():
        return LIB if LIB.exists() else None
    src = Path(root) / SOURCE
    if LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime and LIB.stat().st_mtime >= Path(__file__).stat().st_mtime:
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    nvcc = str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-diag-suppress", "177,550", f"-I{src.parent}", str(src), "-o", str(LIB)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("reference megakernel build failed")
    return LIB


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
