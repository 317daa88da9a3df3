"""Build recipe for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Two shared libraries come out of this file:

* ``oracle/liboracle.so`` -- the C restatement in ``oracle/vbq_oracle.c``.
* ``oracle/_ref/libvbref.so`` -- the reference's own CPU path, compiled straight from
  its sources ``cpp/src/dequant.cpp`` and ``cpp/src/fp16_compat.cpp`` with the
  reference's release flags ``-O3 -DNDEBUG`` (cpp/CMakeLists.txt:177), without the
  reference's build system.  The sources are read where they lie: ``$VB_REF`` when set,
  else a checkout named ``reference`` beside this repository's directory; nothing is
  copied into this repository.  Where neither exists (a machine without the reference
  checkout), only a prebuilt ``.so`` is used.

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
# the same sources with the reference's x86 release flags on an AVX2 host
# (cpp/CMakeLists.txt:177 and :206-208: -O3 -DNDEBUG -mavx2 -mfma); used for timing only,
# and only where the host CPU reports avx2 and fma
REF_AVX2_SO = REF_DIR / "libvbref_avx2.so"
# the reference's GGUF reader (cpp/src/gguf.cpp) behind oracle/ref_gguf_shim.cpp
REF_GGUF_SO = REF_DIR / "libvbref_gguf.so"
GGUF_SHIM = HERE / "ref_gguf_shim.cpp"
# a reference checkout beside this repository's directory, unless $VB_REF names one
DEFAULT_REF = HERE.parent.parent / "reference"


def ref_root() -> Path:
    """The reference checkout: ``$VB_REF``, else ``reference`` beside this repository."""
    return Path(os.environ.get("VB_REF", str(DEFAULT_REF)))


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
    root = ref_root() / "cpp"
    srcs = [root / "src" / "dequant.cpp", root / "src" / "fp16_compat.cpp"]
    if not all(s.exists() for s in srcs):
        return REF_SO if REF_SO.exists() else None
    REF_DIR.mkdir(exist_ok=True)
    for target, extra in ((REF_SO, []), (REF_AVX2_SO, ["-mavx2", "-mfma"])):
        if force or _stale(target, srcs):
            cmd = ["g++", "-O3", "-DNDEBUG", *extra, "-fPIC", "-shared", "-std=c++17",
                   "-I", str(root / "include"), "-I", str(root / "src"),
                   *map(str, srcs), "-o", str(target)]
            subprocess.run(cmd, check=True)
    return REF_SO


def build_ref_gguf(force: bool = False) -> Path | None:
    """Compile the reference's GGUF reader with the C shim into oracle/_ref/libvbref_gguf.so
    (None when neither the sources nor a prebuilt library exist)."""
    root = ref_root() / "cpp"
    srcs = [root / "src" / "gguf.cpp"]
    if not srcs[0].exists():
        return REF_GGUF_SO if REF_GGUF_SO.exists() else None
    REF_DIR.mkdir(exist_ok=True)
    if force or _stale(REF_GGUF_SO, srcs + [GGUF_SHIM]):
        cmd = ["g++", "-O2", "-DNDEBUG", "-fPIC", "-shared", "-std=c++17",
               "-I", str(root / "include"), "-I", str(root / "src"),
               str(GGUF_SHIM), *map(str, srcs), "-o", str(REF_GGUF_SO)]
        subprocess.run(cmd, check=True)
    return REF_GGUF_SO


def host_has_avx2() -> bool:
    """Whether this host's CPU reports AVX2 and FMA (Linux /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return "avx2" in flags and "fma" in flags
    except OSError:
        pass
    return False


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)
    build_ref_gguf(force)


if __name__ == "__main__":
    build_all(force=True)
    print(ORACLE_SO, REF_SO if REF_SO.exists() else "(reference sources absent)")
