"""Generate golden input/output vectors from the reference's own Python code.

Run where the reference checkout is available (it is not on GPU machines):
``python tests/golden/make_golden.py [--reference-dir DIR]``.

The reference's modules import pycuda at module level; pycuda is a GPU-only
dependency that is not installed here, so it is replaced by an empty stub
module before import.  Nothing on the paths used below touches pycuda: the
functions called are pure PyTorch, run on CPU tensors:

* ``pytorch_depthwise_same`` (benchmark/benchmark_shape_sweep_ampere.py:220-239)
  for FWD, with autograd for dX and dK (the reference's validation recipe,
  benchmark/benchmark_pathtile_candidate_sweep.py:153-243), in float32 and
  float64;
* ``reference_depthwise_conv`` (kernels/warp_tiled_ampere.py:901-903), the
  symmetric-padding-then-slice form, which must equal the above;
* ``reference_fp64`` (benchmark/diagnose_dk_correctness.py:44-56), the direct
  FP64 dK formula.

Inputs are seeded CPU tensors (x, k, dy ~ N(0,1); k scaled by 1/sqrt(K) except
for the reference-correctness cases, which use unscaled k as
kernels/warp_tiled_ampere.py:940-942 does).  Output: one compressed .npz per
case plus MANIFEST.json with the shapes, seeds and sha256 of every file.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (case id, B, H, L, K, seed, scale k by 1/sqrt(K))
CASES = [
    # reference correctness cases (kernels/warp_tiled_ampere.py:919-926), small B where large
    ("ref_b2_h4_l16_k8", 2, 4, 16, 8, 0, False),
    ("ref_b4_h8_l31_k16", 4, 8, 31, 16, 0, False),
    ("ref_b8_h16_l48_k24", 8, 16, 48, 24, 0, False),
    ("ref_b4_h64_l48_k48", 4, 64, 48, 48, 0, False),
    ("ref_b2_h128_l48_k48", 2, 128, 48, 48, 0, False),
    # primary and edge shapes of the benchmark, batch reduced
    ("primary_b3_h128_l48_k48", 3, 128, 48, 48, 42, True),
    ("edge_b5_h64_l37_k13", 5, 64, 37, 13, 42, True),
    ("edge_b4_h256_l16_k4", 4, 256, 16, 4, 42, True),
    ("edge_b3_h128_l48_k3", 3, 128, 48, 3, 42, True),
    ("edge_b1_h512_l33_k33", 1, 512, 33, 33, 42, True),
    # degenerate and ragged shapes
    ("deg_b1_h1_l1_k1", 1, 1, 1, 1, 7, True),
    ("deg_b3_h5_l1_k48", 3, 5, 1, 48, 7, True),
    ("deg_b2_h3_l48_k1", 2, 3, 48, 1, 7, True),
    ("deg_b3_h7_l5_k48", 3, 7, 5, 48, 7, True),
    ("deg_b5_h3_l47_k2", 5, 3, 47, 2, 7, True),
    ("odd_b7_h33_l29_k17", 7, 33, 29, 17, 11, True),
    ("odd_b2_h300_l44_k45", 2, 300, 44, 45, 11, True),
    ("odd_b20_h20_l40_k40", 20, 20, 40, 40, 11, True),
]


def _stub_pycuda() -> None:
    pkg = types.ModuleType("pycuda")
    pkg.__path__ = []  # mark as package
    drv = types.ModuleType("pycuda.driver")
    comp = types.ModuleType("pycuda.compiler")
    garr = types.ModuleType("pycuda.gpuarray")

    class _Unavailable:  # any use would be a bug in this script
        def __init__(self, *a, **k):
            raise RuntimeError("pycuda is stubbed for golden-vector generation")

    comp.SourceModule = _Unavailable
    drv.PointerHolderBase = object
    pkg.driver, pkg.compiler, pkg.gpuarray = drv, comp, garr
    sys.modules.update({"pycuda": pkg, "pycuda.driver": drv, "pycuda.compiler": comp,
                        "pycuda.gpuarray": garr})


def _inputs(B, H, L, K, seed, scale):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, H, L, generator=g, dtype=torch.float32)
    k = torch.randn(H, K, generator=g, dtype=torch.float32)
    if scale:
        k = k / (K ** 0.5)
    dy = torch.randn(B, H, L, generator=g, dtype=torch.float32)
    return x, k, dy


def _autograd(fn, x, k, dy):
    xr = x.detach().clone().requires_grad_(True)
    kr = k.detach().clone().requires_grad_(True)
    y = fn(xr, kr)
    gx, gk = torch.autograd.grad(y, (xr, kr), dy)
    return y.detach(), gx.detach(), gk.detach()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference-dir", type=Path, default=HERE.parents[2] / "reference")
    args = ap.parse_args()
    ref = args.reference_dir.resolve()
    if not (ref / "kernels" / "warp_tiled_ampere.py").exists():
        raise SystemExit(f"reference checkout not found at {ref}")
    _stub_pycuda()
    sys.path.insert(0, str(ref))
    torch.set_num_threads(1)
    from benchmark import benchmark_shape_sweep_ampere as sweep  # noqa: E402
    from benchmark import diagnose_dk_correctness as diag  # noqa: E402
    from kernels import warp_tiled_ampere as wta  # noqa: E402

    manifest = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                "reference_functions": [
                    "benchmark/benchmark_shape_sweep_ampere.py:pytorch_depthwise_same",
                    "kernels/warp_tiled_ampere.py:reference_depthwise_conv",
                    "benchmark/diagnose_dk_correctness.py:reference_fp64"],
                "cases": []}
    for cid, B, H, L, K, seed, scale in CASES:
        x, k, dy = _inputs(B, H, L, K, seed, scale)
        y, gx, gk = _autograd(sweep.pytorch_depthwise_same, x, k, dy)
        y64, gx64, gk64_autograd = _autograd(sweep.pytorch_depthwise_same, x.double(), k.double(), dy.double())
        y_sym = wta.reference_depthwise_conv(x, k)
        gk64 = diag.reference_fp64(torch, x, dy, K, 64)
        arrays = {
            "x": x.numpy(), "k": k.numpy(), "dy": dy.numpy(),
            "y": y.numpy(), "gx": gx.numpy(), "gk": gk.numpy(),
            "y64": y64.numpy(), "gx64": gx64.numpy(), "gk64": gk64.numpy(),
        }
        sym_diff = float((y - y_sym).abs().max())
        fp64_diff = float((gk64 - gk64_autograd).abs().max())
        path = HERE / f"{cid}.npz"
        np.savez_compressed(path, **arrays)
        manifest["cases"].append({"id": cid, "B": B, "H": H, "L": L, "K": K, "seed": seed,
                                  "k_scaled": scale, "file": path.name,
                                  "max_abs_sym_minus_same": sym_diff,
                                  "max_abs_dk_fp64_formula_minus_autograd": fp64_diff,
                                  "sha256": hashlib.sha256(path.read_bytes()).hexdigest()})
        print(f"{cid}: y max|sym-asym|={sym_diff:.3e}  gk64 |fp64 formula - fp64 autograd|={fp64_diff:.3e}")
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n", encoding="utf-8")


if __name__ == "__main__":
    main()
