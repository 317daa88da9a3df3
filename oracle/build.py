"""Build recipe for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Two shared libraries come out of this file:

* ``oracle/liboracle.so`` -- the C restatement in ``oracle/vbq_oracle.c``.
* ``oracle/_ref/libvbref.so`` -- the reference's own CPU path, compiled straight from
  its sources ``cpp/src/dequant.cpp`` and ``cpp/src/fp16_compat.cpp`` with the
  reference's release flags ``-O3 -DNDEBUG`` (cpp/CMakeLists.txt:177), without the
  reference's build system.  The sources are read where they lie (``$VB_REF``, default
  the mounted reference checkout); nothing is copied into this repository.  The GPU
  box has no reference checkout, so there only the prebuilt ``.so`` is used.

Run ``python -m oracle.build`` or call :func:`build_all`.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SRC = HERE / "vbq_oracle.c"
ORACLE_SO = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_SO = REF_DIR / "libvbref.so"
DEFAULT_REF = "/root/reference"  # the read-only mount of the build container


def _ref_root() -> Path:
    return Path(os.environ.get("VB_REF", DEFAULT_REF))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def build_oracle(force: bool = False) -> Path:
    """Compile the C restatement.  -ffp-contract=off keeps every multiply and add
    separately rounded, as the reference's scalar x86-64 build evaluates them."""
    if force or _stale(ORACLE_SO, [ORACLE_SRC]):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11",
               str(ORACLE_SRC), "-o", str(ORACLE_SO), "-lm"]
        subprocess.run(cmd, check=True)
    return ORACLE_SO


def build_ref(force: bool = False) -> Path | None:
    """Compile the reference dequant/gemv sources into oracle/_ref/libvbref.so.

    Returns None when the reference checkout is absent (for example on the GPU box,
    which relies on the library built in the container and shipped with the tree)."""
    root = _ref_root() / "cpp"
    srcs = [root / "src" / "dequant.cpp", root / "src" / "fp16_compat.cpp"]
    if not all(s.exists() for s in srcs):
        return REF_SO if REF_SO.exists() else None
    REF_DIR.mkdir(exist_ok=True)
    if force or _stale(REF_SO, srcs):
        cmd = ["g++", "-O3", "-DNDEBUG", "-fPIC", "-shared", "-std=c++17",
               "-I", str(root / "include"), "-I", str(root / "src"),
               *map(str, srcs), "-o", str(REF_SO)]
        subprocess.run(cmd, check=True)
    return REF_SO


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)


if __name__ == "__main__":
    build_all(force=True)
    print(ORACLE_SO, REF_SO if REF_SO.exists() else "(reference sources absent)")
