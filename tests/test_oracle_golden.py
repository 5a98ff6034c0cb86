"""CPU: pin the oracle against golden vectors made by the reference's own code.

The golden files (tests/golden/make_golden.py) hold outputs of the reference's
``pytorch_depthwise_same`` / ``reference_depthwise_conv`` / ``reference_fp64``
on seeded inputs.  The C FP64 oracle and the restated PyTorch path must
reproduce them; only then are they trusted as the checker of the CUDA path.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_cases, golden_manifest, load_golden
from oracle import c_oracle, reference_torch

CASES = golden_cases()
IDS = [c["id"] for c in CASES]


def test_manifest_hashes_match_files():
    for c in golden_manifest()["cases"]:
        data = (GOLDEN / c["file"]).read_bytes()
        assert hashlib.sha256(data).hexdigest() == c["sha256"], c["id"]


def test_reference_functions_agree_in_manifest():
    # The reference's symmetric-pad-then-slice form equals the asymmetric pad
    # form bit for bit, and its FP64 dK formula equals FP64 autograd.
    for c in golden_manifest()["cases"]:
        assert c["max_abs_sym_minus_same"] == 0.0, c["id"]
        assert c["max_abs_dk_fp64_formula_minus_autograd"] < 1e-12, c["id"]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_c_oracle_matches_golden_fp64(case):
    g = load_golden(case)
    y = c_oracle.fwd(g["x"], g["k"])
    gx = c_oracle.dx(g["dy"], g["k"])
    gk = c_oracle.dk(g["dy"], g["x"], case["K"])
    for got, ref in ((y, g["y64"]), (gx, g["gx64"]), (gk, g["gk64"])):
        scale = max(1.0, float(np.abs(ref).max()))
        assert np.abs(got - ref).max() <= 1e-12 * scale


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_torch_restatement_matches_golden_fp32(case):
    g = load_golden(case)
    x, k, dy = (torch.from_numpy(g[n]) for n in ("x", "k", "dy"))
    y, gx, gk = reference_torch.fwd_dx_dk(x, k, dy)
    # Same torch ops on the same inputs; tolerance only covers CPU-kernel
    # differences between machines.
    np.testing.assert_allclose(y.numpy(), g["y"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gx.numpy(), g["gx"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gk.numpy(), g["gk"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fp64_dk_restatement_matches_golden(case):
    g = load_golden(case)
    gk = reference_torch.dk_fp64(torch.from_numpy(g["x"]), torch.from_numpy(g["dy"]), case["K"])
    np.testing.assert_allclose(gk.numpy(), g["gk64"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_golden_fp32_outputs_within_spec_of_fp64(case):
    # The reference's own FP32 outputs satisfy the parity bar against FP64,
    # so the bar (1e-5 FWD/dX, 1e-4 relative dK) is attainable in FP32.
    g = load_golden(case)
    np.testing.assert_allclose(g["y"], g["y64"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(g["gx"], g["gx64"], rtol=1e-5, atol=1e-5)
    scale = float(np.abs(g["gk64"]).max())
    np.testing.assert_allclose(g["gk"], g["gk64"], rtol=1e-4, atol=1e-4 * scale)


def test_oracle_catches_a_planted_error():
    # A deliberately wrong oracle output (one tap shifted) must fail the check.
    case = next(c for c in CASES if c["id"].startswith("primary"))
    g = load_golden(case)
    y = c_oracle.fwd(g["x"], np.roll(g["k"], 1, axis=1))
    assert np.abs(y - g["y64"]).max() > 1e-2


def test_make_inputs_seeded_and_scaled():
    x1, k1, d1 = reference_torch.make_inputs(4, 8, 16, 9, seed=42)
    x2, k2, d2 = reference_torch.make_inputs(4, 8, 16, 9, seed=42)
    assert torch.equal(x1, x2) and torch.equal(k1, k2) and torch.equal(d1, d2)
    big = reference_torch.make_inputs(64, 128, 48, 48, seed=1)[1]
    assert abs(float(big.std()) * 48 ** 0.5 - 1.0) < 0.05


def test_case_seed_matches_reference_rule():
    import zlib

    cid = "main_b16384_h128_l48_k48"
    assert reference_torch.case_seed(42, cid) == 42 + zlib.crc32(cid.encode())
