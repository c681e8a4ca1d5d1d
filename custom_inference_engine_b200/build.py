"""Builds the two native libraries of the package, in-tree, for sm_100a.

* ``libcie_attention.so`` -- the CUDA kernels and their C ABI
  (``include/cie_attention.h``, ``include/cie_model_ops.h``), compiled by nvcc
  from ``csrc/cie_unity.cu`` and ``csrc/model_ops.cu``; the CUDA runtime is
  linked statically and its symbols are not exported.
* ``_cie_torch_ops.so`` -- the ``inference::*`` torch ops
  (``csrc/torch_ops.cpp``) linked against the library above
  (rpath ``$ORIGIN``), built with ``torch.utils.cpp_extension``.

Both land next to this file so they travel with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libcie_attention.so"
OPS = PKG / "_cie_torch_ops.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _cu_deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    """Two objects linked into one library: the attention kernels
    (``cie_unity.cu``, --use_fast_math) and the Qwen2 body kernels
    (``model_ops.cu``, IEEE division and library expf / rsqrtf, so that they
    round like torch's own kernels)."""
    if not force and not _stale(LIB, _cu_deps()):
        return LIB
    bdir = PKG / "_build"
    bdir.mkdir(exist_ok=True)
    common = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
              "-I", str(INCLUDE), "-I", str(CSRC)]
    if verbose:
        common.insert(1, "-Xptxas=-v")
    objs = [(CSRC / "cie_unity.cu", ["--use_fast_math"]), (CSRC / "model_ops.cu", [])]
    out = []
    for src, extra in objs:
        obj = bdir / (src.stem + ".o")
        cmd = [*common, *extra, "-c", "-o", str(obj), str(src)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        out.append(str(obj))
    cmd = [_nvcc(), *ARCH, "-shared", "-Xlinker", "--exclude-libs,ALL", "-o", str(LIB) + ".tmp",
           *out]
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def build_ops(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / "torch_ops.cpp", *sorted(INCLUDE.glob("*.h")), LIB]
    if not force and not _stale(OPS, deps):
        return OPS
    # torch.utils.cpp_extension.load also loads the library into the calling
    # process, which would register the inference:: namespace a second time when
    # the package later loads its in-tree copy: compile in a child process.
    subprocess.run([sys.executable, "-c",
                    "import sys; sys.path.insert(0, %r); "
                    "from custom_inference_engine_b200 import build; "
                    "build._compile_ops(%r)" % (str(PKG.parent), verbose)], check=True)
    return OPS


def _compile_ops(verbose: bool = False) -> None:
    from torch.utils.cpp_extension import load
    bdir = PKG / "_build"
    bdir.mkdir(exist_ok=True)
    load(name="_cie_torch_ops", sources=[str(CSRC / "torch_ops.cpp")],
         extra_include_paths=[str(INCLUDE)],
         extra_cflags=["-O3"],
         # '$$' survives ninja, the single quotes survive the shell: the
         # runpath is literally $ORIGIN (package dir) and $ORIGIN/.. (from _build)
         extra_ldflags=[f"-L{PKG}", "-lcie_attention",
                        "'-Wl,-rpath,$$ORIGIN:$$ORIGIN/..'"],
         build_directory=str(bdir), with_cuda=True, is_python_module=False,
         verbose=verbose)
    shutil.copy2(bdir / "_cie_torch_ops.so", str(OPS) + ".tmp")
    os.replace(str(OPS) + ".tmp", OPS)


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ops(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
