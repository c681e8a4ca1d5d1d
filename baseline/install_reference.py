"""Place an unmodified copy of the reference engine's Python tree in ``baseline/_ref``.

The reference (eteboun/custom_inference_engine) is a loose tree of Python
packages with no ``setup.py`` or ``pyproject.toml``, so ``pip install --target``
cannot install it; this script copies its ``*.py`` files instead, byte for byte,
keeping the package layout (``scheduler/``, ``piecewise/``, ``attn/``,
``kv_cache/``, ``kernels/``, ...). ``baseline/_ref`` is git-ignored: the copy is
test infrastructure, never part of the package, and nothing under
``custom_inference_engine_b200/`` imports it. Tests use it to run the reference's
own graph modules (``scheduler/decode_module.py``, ``scheduler/mixed_module.py``,
``piecewise/``) over this package's ops, and skip when it is absent.

Usage: ``python baseline/install_reference.py [SOURCE]`` (SOURCE defaults to
``$CIE_REFERENCE_SOURCE``). Exits 0 without copying when SOURCE does not exist.
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

DEST = Path(__file__).resolve().parent / "_ref"
PACKAGES = ("attn", "kv_cache", "kernels", "scheduler", "piecewise", "benchmark",
            "feature_bench", "vllm_baseline")


def install(source: Path, dest: Path = DEST) -> int:
    """Copy the reference's Python files from ``source`` to ``dest``; returns the file count."""
    source = Path(source)
    if not source.is_dir():
        return 0
    if dest.exists():
        shutil.rmtree(dest)
    n = 0
    for top in source.glob("*.py"):
        dest.mkdir(parents=True, exist_ok=True)
        shutil.copy2(top, dest / top.name)
        n += 1
    for pkg in PACKAGES:
        for f in sorted((source / pkg).rglob("*.py")):
            out = dest / f.relative_to(source)
            out.parent.mkdir(parents=True, exist_ok=True)
            shutil.copy2(f, out)
            n += 1
    return n


def main() -> int:
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CIE_REFERENCE_SOURCE", "")
    if not src or not Path(src).is_dir():
        print(f"install_reference: no reference tree at {src!r}; nothing copied")
        return 0
    n = install(Path(src))
    print(f"install_reference: {n} files -> {DEST}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
