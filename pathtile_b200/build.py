"""Build ``pathtile_b200/libpathtile_b200.so`` (sm_100a) in-tree with nvcc.

Every ``.cu`` unit under ``pathtile_b200/csrc`` is compiled in parallel for
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared library
with a static CUDA runtime, so the file is self-contained apart from the
driver.  Rebuilds only when a source or header is newer than the library.

Usage: ``python -m pathtile_b200.build [--force] [--verbose-ptxas]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libpathtile_b200.so"
OBJ_DIR = ROOT / "_build" / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build pathtile_b200")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}\n{res.stdout}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library; returns its path."""
    if not force and not verbose_ptxas and not needs_build():
        return LIB
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    jobs = jobs or max(1, min(len(srcs), os.cpu_count() or 1))
    logs: list[str] = []
    objs: list[Path] = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), srcs):
            objs.append(obj)
            if log.strip():
                logs.append(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}\n{res.stdout}")
    os.replace(tmp, LIB)
    if verbose_ptxas:
        sys.stderr.write("\n".join(logs))
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)


if __name__ == "__main__":
    main()
