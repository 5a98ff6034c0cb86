"""TEST INFRASTRUCTURE ONLY -- build recipe of the oracle libraries.

* ``liboracle.so`` from ``pt_oracle.c`` (gcc, OpenMP): the FP64 CPU checker.
* ``_ref/libref_warptile.so`` (only where the reference checkout is present):
  the reference's own warp-tiled CUDA kernels compiled for sm_100a.  The kernel
  text is read from the reference's kernels/warp_tiled_ampere.py (the
  CUDA_TEMPLATE string, located with ``ast`` as the reference itself does in
  benchmark/benchmark_dk_packing.py:44-57), its launch constants substituted
  with the reference defaults, and written to ``_ref/`` (git-ignored, so the
  reference source never enters this repository's history).  It is compiled
  with the reference's own nvcc options (kernels/warp_tiled_ampere.py:675-685)
  together with ``ref_shim.cu``.  Built artefacts travel with the working tree
  to GPU machines, where the reference checkout does not exist.

Usage: ``python -m oracle.build_oracle``.
"""
from __future__ import annotations

import ast
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
C_LIB = HERE / "liboracle.so"
REF_LIB = REF_OUT / "libref_warptile.so"


def reference_dir() -> Path:
    env = os.environ.get("PATHTILE_REFERENCE_DIR")
    return Path(env) if env else HERE.parents[1] / "reference"


def build_c_oracle(force: bool = False) -> Path:
    src = HERE / "pt_oracle.c"
    if not force and C_LIB.exists() and C_LIB.stat().st_mtime >= src.stat().st_mtime:
        return C_LIB
    tmp = C_LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fopenmp", "-shared", "-fPIC", str(src), "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    os.replace(tmp, C_LIB)
    return C_LIB


def _cuda_template(path: Path) -> str:
    tree = ast.parse(path.read_text(encoding="utf-8"))
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id == "CUDA_TEMPLATE" for t in node.targets
        ):
            return ast.literal_eval(node.value)
    raise RuntimeError(f"CUDA_TEMPLATE not found in {path}")


def build_reference_kernels(force: bool = False) -> Path | None:
    """Compile the reference's kernels for sm_100a; None when the reference is absent."""
    src = reference_dir() / "kernels" / "warp_tiled_ampere.py"
    if not src.exists():
        return None
    shim = HERE / "ref_shim.cu"
    if (not force and REF_LIB.exists() and REF_LIB.stat().st_mtime >= src.stat().st_mtime
            and REF_LIB.stat().st_mtime >= shim.stat().st_mtime):
        return REF_LIB
    REF_OUT.mkdir(parents=True, exist_ok=True)
    text = (_cuda_template(src).replace("__WARPS_PER_BLOCK__", "16")
            .replace("__BWDK_BTILE__", "64").replace("__BWDK_BLOCK__", "128"))
    gen = REF_OUT / "ref_warptile_kernels.cu"
    gen.write_text(text, encoding="utf-8")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-ftz=true",
           "-prec-div=false", "-prec-sqrt=false", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           f'-DREF_KERNELS_FILE="{gen}"', str(shim), "-o", str(REF_LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference kernel build failed:\n{res.stderr}")
    return REF_LIB


def main() -> None:
    print(build_c_oracle(force=True))
    print(build_reference_kernels(force=True))


if __name__ == "__main__":
    main()
