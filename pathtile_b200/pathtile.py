"""PathTile offline launch-configuration selection, re-run for B200.

The reference sweeps launch candidates per path on 20 tuning shapes, picks
per path the candidate with the minimum SUM of mean latency over those shapes
(ties to the smaller value), freezes it, and scores it on held-out shapes by
regret = frozen_total / oracle_total - 1, where total = FWD + dX + dK and the
oracle picks the best candidate per shape and path
(benchmark/benchmark_pathtile_candidate_sweep.py:485-560,
scripts/aggregate_pathtile_results.py:222-240 and :376-420).

B200 candidate axes are runtime values of the native library (no
recompilation): rows per tile (one thread per row), TMA ring depth and
persistent CTAs per SM, per path.  Every candidate is validated before it is
timed, at a batch of at most 128, against PyTorch's own conv1d on the GPU with
TF32 off (the reference's validation recipe, :153-243).

A second axis is the engine of FWD and dX: the CUDA-core FFMA kernels (the
candidates above) or the tcgen05 tensor-core kernels (FP32-accurate 3xTF32
split, L % 4 == 0 only, no launch knobs).  The engine sweep times, per
shape, the frozen FFMA launch against the tensor engine (both validated the
same way, visits alternating); per path and intensity class the engine with
the smaller summed latency over that class's shapes is frozen -- the same
selection rule applied to the engine axis.

Modes:
  run        sweep one preset, one trial -> <out>/trialN/raw.csv, summary.csv
  aggregate  average trials, select the frozen policy -> frozen_config.json and
             the C header pathtile_b200/csrc/pt_frozen_config.h (with
             --engines, the engine table of an engine sweep goes into it too)
  regret     score the frozen policy on a held-out sweep against its per-shape oracle
  engines    engine sweep of one preset -> <out>/engines.csv, engine_policy.json
  backward   backward-kernel sweep of one preset -> <out>/backward.csv; selects
             the backward policy (backward_policy.json, --write-header puts it
             into the header) or, with --bwd-policy, scores a frozen one

The backward axis is the kernel pt_dx_dk runs -- dX then dK, the tensor-core
fused kernel (with or without helper CTAs for the tail blocks: the most
channels one helper may own), or the CUDA-core fused kernel -- frozen per
intensity class as a policy (kernel mode, helper limit) with the same rule:
the policy with the minimum summed latency over the class's tuning shapes,
ties to the smaller policy.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import statistics
import time
import zlib
from dataclasses import asdict, dataclass
from pathlib import Path

PATHS = ("fwd", "bwd_input", "bwd_weight")
ROWS = (64, 128, 256)
STAGES = (2, 3, 4)
CTAS = (1, 2, 3, 4)
TPRS = (1, 2)
HEADER = Path(__file__).resolve().parent / "csrc" / "pt_frozen_config.h"


@dataclass(frozen=True)
class ShapeCase:
    config_id: str
    B: int
    H: int
    L: int
    K: int
    sweep_group: str

    def validate(self) -> None:
        if min(self.B, self.H, self.L, self.K) <= 0:
            raise ValueError(f"All dimensions must be positive: {self}")
        if self.L > 48 or self.K > 48:
            raise ValueError(f"{self.config_id}: kernels require L<=48 and K<=48")


def _c(cid: str, B: int, H: int, L: int, K: int, group: str) -> ShapeCase:
    return ShapeCase(cid, B, H, L, K, group)


# The reference's 20 tuning shapes and 10 held-out shapes
# (benchmark/benchmark_shape_sweep_ampere.py:79-178), same ids and sizes.
PATHTILE_TRAIN_CASES = [
    _c("main_b16384_h128_l48_k48", 16384, 128, 48, 48, "main"),
    _c("batch_b2048_h128_l48_k48", 2048, 128, 48, 48, "batch"),
    _c("batch_b8192_h128_l48_k48", 8192, 128, 48, 48, "batch"),
    _c("channel_b8192_h64_l48_k48", 8192, 64, 48, 48, "channel"),
    _c("channel_b8192_h256_l48_k48", 8192, 256, 48, 48, "channel"),
    _c("sequence_b8192_h128_l16_k16", 8192, 128, 16, 16, "sequence"),
    _c("sequence_b8192_h128_l24_k24", 8192, 128, 24, 24, "sequence"),
    _c("sequence_b8192_h128_l32_k32", 8192, 128, 32, 32, "sequence"),
    _c("kernel_b8192_h128_l48_k8", 8192, 128, 48, 8, "kernel"),
    _c("kernel_b8192_h128_l48_k24", 8192, 128, 48, 24, "kernel"),
    _c("mix_b4096_h64_l32_k16", 4096, 64, 32, 16, "mixed"),
    _c("mix_b4096_h256_l48_k24", 4096, 256, 48, 24, "mixed"),
    _c("mix_b2048_h64_l24_k8", 2048, 64, 24, 8, "mixed"),
    _c("mix_b2048_h256_l32_k32", 2048, 256, 32, 32, "mixed"),
    _c("mix_b8192_h64_l32_k24", 8192, 64, 32, 24, "mixed"),
    _c("mix_b8192_h256_l24_k16", 8192, 256, 24, 16, "mixed"),
    _c("mix_b16384_h64_l48_k8", 16384, 64, 48, 8, "mixed"),
    _c("mix_b16384_h256_l16_k16", 16384, 256, 16, 16, "mixed"),
    _c("mix_b16384_h128_l32_k24", 16384, 128, 32, 24, "mixed"),
    _c("mix_b4096_h128_l48_k32", 4096, 128, 48, 32, "mixed"),
]

PATHTILE_HOLDOUT_CASES = [
    _c("holdout_b4096_h96_l40_k20", 4096, 96, 40, 20, "holdout"),
    _c("holdout_b12288_h192_l40_k32", 12288, 192, 40, 32, "holdout"),
    _c("holdout_b12288_h96_l20_k12", 12288, 96, 20, 12, "holdout"),
    _c("holdout_b4096_h192_l28_k24", 4096, 192, 28, 24, "holdout"),
    _c("holdout_b12288_h64_l40_k40", 12288, 64, 40, 40, "holdout"),
    _c("holdout_b4096_h256_l20_k16", 4096, 256, 20, 16, "holdout"),
    _c("holdout_b2048_h192_l40_k32", 2048, 192, 40, 32, "holdout"),
    _c("holdout_b12288_h128_l28_k20", 12288, 128, 28, 20, "holdout"),
    _c("holdout_b4096_h64_l40_k12", 4096, 64, 40, 12, "holdout"),
    _c("holdout_b12288_h256_l32_k24", 12288, 256, 32, 24, "holdout"),
]

# Held-out sweep of this build's specification: B x H x (L, K), K <= L.
SWEEP_LK = [(24, 8), (24, 16), (32, 8), (32, 16), (32, 32), (48, 8), (48, 16), (48, 32), (48, 48)]
HELDOUT_SWEEP_CASES = [
    _c(f"sweep_b{B}_h{H}_l{L}_k{K}", B, H, L, K, "sweep")
    for B in (4096, 16384, 32768) for H in (64, 128, 256) for (L, K) in SWEEP_LK
]

EDGE_CASES = [
    _c("edge_b4096_h64_l37_k13", 4096, 64, 37, 13, "edge"),
    _c("edge_b8192_h256_l16_k4", 8192, 256, 16, 4, "edge"),
    _c("edge_b16384_h128_l48_k3", 16384, 128, 48, 3, "edge"),
    _c("edge_b2048_h512_l33_k33", 2048, 512, 33, 33, "edge"),
]

SMOKE_CASES = [
    _c("smoke_b64_h8_l16_k8", 64, 8, 16, 8, "smoke"),
    _c("smoke_b128_h16_l48_k48", 128, 16, 48, 48, "smoke"),
]

PRESETS = {
    "pathtile-train": PATHTILE_TRAIN_CASES,
    "pathtile-holdout": PATHTILE_HOLDOUT_CASES,
    "heldout-sweep": HELDOUT_SWEEP_CASES,
    "edge": EDGE_CASES,
    "smoke": SMOKE_CASES,
}


def cases_for_preset(preset: str) -> list[ShapeCase]:
    if preset not in PRESETS:
        raise ValueError(f"Unknown preset: {preset}")
    cases = list(PRESETS[preset])
    for c in cases:
        c.validate()
    return cases


def case_seed(base_seed: int, case: ShapeCase) -> int:
    """base + crc32(config id), as benchmark_pathtile_candidate_sweep.py:109-110."""
    return int(base_seed + zlib.crc32(case.config_id.encode("utf-8")))


CLASSES = ("light", "medium", "heavy")


def in_range_pairs(L: int, K: int) -> int:
    """(t, j) pairs with 0 <= t+j-K//2 < L: the FMAs one row needs."""
    pad = K // 2
    return sum(max(0, min(L, L + pad - j) - max(0, pad - j)) for j in range(K))


def intensity_class(L: int, K: int) -> str:
    """Arithmetic-intensity class of a shape: in-range FMAs per output element
    below 12 -> light (memory-bound), below 24 -> medium, else heavy (near the
    FP32 ridge).  The native library computes the same class (pt_api.cu)."""
    f = in_range_pairs(L, K) / L
    return "light" if f < 12 else ("medium" if f < 24 else "heavy")


ENGINES = ("ffma", "tensor")
ENGINE_PATHS = ("fwd", "bwd_input")  # dK has no tensor-core kernel


def tensor_applicable(L: int) -> bool:
    """Shapes the frozen table may send to the tensor engine: L % 4 == 0 (TMA
    boxes of 16 or 32 floats) and 48 % L == 0, so that every tile row is a
    full 48-column super-row (one L = 48 channel or 48 / L packed channels);
    partially filled tiles stay on the FFMA kernels, which measured faster."""
    return L % 4 == 0 and 48 % L == 0


def candidates() -> list[tuple[int, int, int, int]]:
    return [(r, s, c, t) for t in TPRS for r in ROWS for s in STAGES for c in CTAS]


def candidate_id(c: tuple) -> str:
    return f"r{c[0]}s{c[1]}c{c[2]}t{c[3]}"


# ---------------------------------------------------------------------------
# Selection logic (pure; unit-tested on CPU)
# ---------------------------------------------------------------------------
def _cand(row: dict) -> tuple[int, int, int, int]:
    """(rows, stages, ctas_per_sm, threads_per_row) of a summary row."""
    return (int(row["rows"]), int(row["stages"]), int(row["ctas_per_sm"]), int(row.get("threads_per_row") or 1))


def _class_of(row: dict) -> str:
    return intensity_class(int(row["L"]), int(row["K"]))


def select_policy(summary: list[dict], per_class: bool = False) -> dict[str, dict[str, tuple[int, int, int]]]:
    """The frozen policy.  Default (the reference's rule): per path, the
    candidate with the minimum sum over all tuning shapes of mean_ms, used for
    every intensity class.  With per_class, the same rule within each class's
    tuning shapes (a class without shapes inherits from the nearest class that
    has some, medium first).  Ties go to the smaller candidate tuple;
    candidates missing any shape of the set (invalid or failed) are not
    eligible."""
    chosen: dict[str, dict[str, tuple[int, int, int]]] = {}
    for path in PATHS:
        chosen[path] = {}
        for cls in (CLASSES if per_class else ("all",)):
            rows = [r for r in summary if r["phase"] == path and (not per_class or _class_of(r) == cls)]
            shapes = {r["config_id"] for r in rows}
            if not shapes:
                continue
            totals: dict[tuple[int, int, int], float] = {}
            seen: dict[tuple[int, int, int], set] = {}
            for r in rows:
                c = _cand(r)
                totals[c] = totals.get(c, 0.0) + float(r["mean_ms"])
                seen.setdefault(c, set()).add(r["config_id"])
            eligible = [(t, c) for c, t in totals.items() if seen[c] == shapes]
            if not eligible:
                raise ValueError(f"No candidate covers every {cls} shape for {path}")
            chosen[path][cls] = min(eligible)[1]
        if not chosen[path]:
            raise ValueError(f"No tuning shapes for {path}")
        if not per_class:
            chosen[path] = {cls: chosen[path]["all"] for cls in CLASSES}
            continue
        for cls in CLASSES:
            if cls not in chosen[path]:
                for alt in ("medium", "heavy", "light"):
                    if alt in chosen[path]:
                        chosen[path][cls] = chosen[path][alt]
                        break
    return chosen


def oracle_totals(summary: list[dict]) -> dict[str, dict[str, float]]:
    """Per shape: best mean_ms per path over all candidates."""
    best: dict[str, dict[str, float]] = {}
    for r in summary:
        d = best.setdefault(r["config_id"], {})
        v = float(r["mean_ms"])
        if r["phase"] not in d or v < d[r["phase"]]:
            d[r["phase"]] = v
    return best


def regret_table(summary: list[dict], policy: dict[str, dict[str, tuple[int, int, int]]]) -> list[dict]:
    """Per shape: frozen total, oracle total and regret (frozen/oracle - 1)."""
    lookup = {}
    cls_of = {}
    for r in summary:
        lookup[(r["config_id"], r["phase"], *_cand(r))] = float(r["mean_ms"])
        cls_of[r["config_id"]] = _class_of(r)
    best = oracle_totals(summary)
    rows = []
    for cid in sorted(best):
        cls = cls_of[cid]
        frozen = sum(lookup[(cid, p, *policy[p][cls])] for p in PATHS)
        oracle = sum(best[cid][p] for p in PATHS)
        rows.append({"config_id": cid, "class": cls, "frozen_total_ms": frozen, "oracle_total_ms": oracle,
                     "regret_pct": 100.0 * (frozen / oracle - 1.0)})
    return rows


# ---------------------------------------------------------------------------
# Selector baselines (the reference's scripts/evaluate_selector_baselines.py):
# static policies scored against the per-shape oracle on a shape set.
# ---------------------------------------------------------------------------
# The reference runtime's defaults (WARPS_PER_BLOCK = 4 -> 128 rows, BWDK_BLOCK,
# kernels/warp_tiled_ampere.py:668-672) on this library's candidate axes.
DEFAULT_POLICY = {"fwd": (128, 3, 2, 1), "bwd_input": (128, 3, 2, 1), "bwd_weight": (128, 2, 2, 1)}


def majority_winner_policy(summary: list[dict]) -> dict[str, tuple[int, int, int, int]]:
    """Per path, the candidate that is fastest on the most shapes (per-shape ties
    to the smaller candidate, then most wins, ties to the smaller candidate)."""
    policy = {}
    for path in PATHS:
        best: dict[str, tuple[float, tuple]] = {}
        for r in summary:
            if r["phase"] != path:
                continue
            key = (float(r["mean_ms"]), _cand(r))
            if r["config_id"] not in best or key < best[r["config_id"]]:
                best[r["config_id"]] = key
        if not best:
            raise ValueError(f"No rows for {path}")
        wins: dict[tuple, int] = {}
        for _, cand in best.values():
            wins[cand] = wins.get(cand, 0) + 1
        policy[path] = min(wins, key=lambda c: (-wins[c], c))
    return policy


def evaluate_baselines(train: list[dict], evalset: list[dict]) -> tuple[list[dict], dict]:
    """Per shape of `evalset`: total FWD + dX + dK latency of each static policy
    chosen on `train` -- default, global (the frozen PathTile rule), majority
    winner -- and of a uniformly random static candidate (expected latency: the
    mean over candidates, per path), against the per-shape oracle."""
    global_pol = select_policy(train)
    policies = {
        "default": DEFAULT_POLICY,
        "global": {p: global_pol[p]["medium"] for p in PATHS},
        "majority_winner": majority_winner_policy(train),
    }
    lookup: dict[tuple, float] = {}
    per_path: dict[tuple, list[float]] = {}
    for r in evalset:
        lookup[(r["config_id"], r["phase"], *_cand(r))] = float(r["mean_ms"])
        per_path.setdefault((r["config_id"], r["phase"]), []).append(float(r["mean_ms"]))
    best = oracle_totals(evalset)
    rows = []
    for cid in sorted(best):
        if any(p not in best[cid] for p in PATHS):
            continue
        oracle = sum(best[cid][p] for p in PATHS)
        row = {"config_id": cid, "oracle_total_ms": oracle}
        for name, pol in policies.items():
            keys = [(cid, p, *pol[p]) for p in PATHS]
            total = sum(lookup[k] for k in keys) if all(k in lookup for k in keys) else float("nan")
            row[f"{name}_total_ms"] = total
            row[f"{name}_regret_pct"] = 100.0 * (total / oracle - 1.0)
        rnd = sum(statistics.mean(per_path[(cid, p)]) for p in PATHS)
        row["random_fixed_total_ms"] = rnd
        row["random_fixed_regret_pct"] = 100.0 * (rnd / oracle - 1.0)
        rows.append(row)
    summary = {"shapes": len(rows),
               "policies": {name: {p: list(c) for p, c in pol.items()} for name, pol in policies.items()}}
    for name in (*policies, "random_fixed"):
        vals = [r[f"{name}_regret_pct"] for r in rows if r[f"{name}_regret_pct"] == r[f"{name}_regret_pct"]]
        if not vals:
            continue
        summary[name] = {
            "mean_regret_pct": statistics.mean(vals),
            "geomean_regret_pct": 100.0 * (math.exp(statistics.mean(math.log1p(v / 100.0) for v in vals)) - 1.0),
            "max_regret_pct": max(vals),
            "within_2pct": sum(v <= 2.0 for v in vals),
            "shapes": len(vals),
        }
    return rows, summary


def select_engines(rows: list[dict]) -> dict[str, dict[str, str]]:
    """Engine per path and intensity class from engine-sweep rows (config_id,
    phase, engine, L, K, mean_ms): "tensor" where its summed latency over the
    class's shapes (those measured on both engines) is strictly smaller than
    the FFMA kernels', else "ffma"; dK and classes without shapes stay "ffma"."""
    out: dict[str, dict[str, str]] = {p: {c: "ffma" for c in CLASSES} for p in PATHS}
    times: dict[tuple, float] = {}
    cls_of: dict[str, str] = {}
    for r in rows:
        times[(r["config_id"], r["phase"], r["engine"])] = float(r["mean_ms"])
        cls_of[r["config_id"]] = _class_of(r)
    for path in ENGINE_PATHS:
        for cls in CLASSES:
            both = [cid for cid, c in cls_of.items() if c == cls
                    and (cid, path, "ffma") in times and (cid, path, "tensor") in times]
            if not both:
                continue
            tf = sum(times[(cid, path, "ffma")] for cid in both)
            tt = sum(times[(cid, path, "tensor")] for cid in both)
            out[path][cls] = "tensor" if tt < tf else "ffma"
    return out


def engine_regret(rows: list[dict], engines: dict[str, dict[str, str]]) -> list[dict]:
    """Per shape: FWD + dX time of the frozen engines vs the faster engine per path."""
    times: dict[tuple, float] = {}
    cls_of: dict[str, str] = {}
    for r in rows:
        times[(r["config_id"], r["phase"], r["engine"])] = float(r["mean_ms"])
        cls_of[r["config_id"]] = _class_of(r)
    out = []
    for cid in sorted(cls_of):
        cls = cls_of[cid]
        if not all((cid, p, e) in times for p in ENGINE_PATHS for e in ENGINES):
            continue
        frozen = sum(times[(cid, p, engines[p][cls])] for p in ENGINE_PATHS)
        best = sum(min(times[(cid, p, e)] for e in ENGINES) for p in ENGINE_PATHS)
        ffma = sum(times[(cid, p, "ffma")] for p in ENGINE_PATHS)
        out.append({"config_id": cid, "class": cls, "frozen_ms": frozen, "best_ms": best, "ffma_ms": ffma,
                    "regret_pct": 100.0 * (frozen / best - 1.0), "gain_vs_ffma_pct": 100.0 * (ffma / frozen - 1.0)})
    return out


# ---------------------------------------------------------------------------
# Backward-kernel axis (pt_launch_opts.bwd_kernel / helper_channels)
# ---------------------------------------------------------------------------
BWD_KINDS = ("separate", "tensor_fused", "ffma_fused")
HELPER_LIMITS = (0, 2, 4, 8)
# Candidate policies (bwd_kernel, helper_channels): PT_BWD_SEPARATE,
# PT_BWD_TENSOR_FUSED, PT_BWD_FFMA_FUSED, PT_BWD_ANY_FUSED.
BWD_POLICIES = ([(0, 0)] + [(1, h) for h in HELPER_LIMITS] + [(2, 0)] + [(3, h) for h in HELPER_LIMITS])


def bwd_policy_id(pol: tuple[int, int]) -> str:
    return f"k{pol[0]}h{pol[1]}"


def _bwd_rows_by_shape(rows: list[dict]) -> dict[str, dict]:
    """config_id -> {"class": ..., "time": {policy: ms}} from backward-sweep rows
    (one row per measured variant, listing the policies that run it)."""
    shapes: dict[str, dict] = {}
    for r in rows:
        d = shapes.setdefault(r["config_id"], {"class": _class_of(r), "time": {}})
        for pid in str(r["policies"]).split(";"):
            if pid:
                d["time"][pid] = float(r["mean_ms"])
    return shapes


def select_backward(rows: list[dict]) -> dict[str, tuple[int, int]]:
    """Per intensity class, the policy with the minimum summed latency over the
    class's shapes (ties to the smaller policy); policies missing any of the
    class's shapes are not eligible; a class without shapes inherits from the
    nearest class that has some (medium first)."""
    shapes = _bwd_rows_by_shape(rows)
    chosen: dict[str, tuple[int, int]] = {}
    for cls in CLASSES:
        members = [d for d in shapes.values() if d["class"] == cls]
        if not members:
            continue
        totals = []
        for pol in BWD_POLICIES:
            pid = bwd_policy_id(pol)
            if all(pid in d["time"] for d in members):
                totals.append((sum(d["time"][pid] for d in members), pol))
        if totals:
            chosen[cls] = min(totals)[1]
    for cls in CLASSES:
        if cls not in chosen:
            for alt in ("medium", "heavy", "light"):
                if alt in chosen:
                    chosen[cls] = chosen[alt]
                    break
    if not chosen:
        raise ValueError("no backward-sweep rows to select from")
    return chosen


def backward_regret(rows: list[dict], policy: dict[str, tuple[int, int]]) -> list[dict]:
    """Per shape: backward time of the frozen policy, of the per-shape best
    variant, and of dX then dK."""
    out = []
    for cid, d in sorted(_bwd_rows_by_shape(rows).items()):
        pid = bwd_policy_id(policy[d["class"]])
        if pid not in d["time"]:
            continue
        frozen = d["time"][pid]
        best = min(d["time"].values())
        sep = d["time"].get(bwd_policy_id((0, 0)))
        out.append({"config_id": cid, "class": d["class"], "frozen_ms": frozen, "best_ms": best,
                    "separate_ms": sep, "regret_pct": 100.0 * (frozen / best - 1.0),
                    "gain_vs_separate_pct": (100.0 * (sep / frozen - 1.0)) if sep else None})
    return out


def apply_backward_to_header(text: str, policy: dict[str, tuple[int, int]]) -> str:
    """Rewrite only the kFrozenBwd table of an existing frozen-config header."""
    start = text.index("constexpr BwdChoice kFrozenBwd[3] = {")
    end = text.index("};", start) + 2
    rows = ["constexpr BwdChoice kFrozenBwd[3] = {"]
    for cls in CLASSES:
        rows.append("    {%d, %d},  // %s" % (policy[cls][0], policy[cls][1], cls))
    rows.append("};")
    return text[:start] + "\n".join(rows) + text[end:]


def _header_backward_block(text: str | None) -> list[str]:
    """The kFrozenBwd block of an existing header (kept when the launch table is
    rewritten), or the default: any fused kernel, helpers owning <= 4 channels."""
    if text and "constexpr BwdChoice kFrozenBwd[3] = {" in text:
        start = text.index("// kFrozenBwd[class]:")
        end = text.index("};", text.index("constexpr BwdChoice kFrozenBwd[3] = {")) + 2
        return text[start:end].split("\n")
    return ["// kFrozenBwd[class]: the kernel pt_dx_dk runs (PT_BWD_*) and the most channels",
            "// a helper CTA of the tensor-core fused kernel may own (0: no helpers).",
            "struct BwdChoice {", "  int kernel;", "  int helper_channels;", "};",
            "constexpr BwdChoice kFrozenBwd[3] = {", "    {3, 4},  // light", "    {3, 4},  // medium",
            "    {3, 4},  // heavy", "};"]


def render_header(policy: dict[str, dict[str, tuple[int, int, int]]], source: str,
                  engines: dict[str, dict[str, str]] | None = None) -> str:
    lines = [
        "// pt_frozen_config.h -- launch configuration per path and intensity class, frozen offline.",
        "//",
        "// Written by `python -m pathtile_b200.pathtile --mode aggregate --write-header`:",
        "// per path and per arithmetic-intensity class (in-range FMAs per output",
        "// element: light < 12 <= medium < 24 <= heavy), the candidate (rows per tile,",
        "// ring stages, CTAs per SM, threads per row) with the minimum sum of mean latency over that",
        "// class's tuning shapes, ties to the smaller candidate -- the reference's",
        "// selection rule (scripts/aggregate_pathtile_results.py:222-240) applied per",
        "// class.  Deployment looks the class up; it does no per-shape search.",
        "#pragma once",
        "",
        "namespace pt {",
        "",
        "struct LaunchCfg {",
        "  int rows;         // rows per tile = threads doing math per CTA (32..256)",
        "  int stages;       // shared-memory ring depth (2..4)",
        "  int ctas_per_sm;  // persistent CTAs per SM (1..4), clamped by occupancy",
        "  int tpr;          // consumer threads per row (1 or 2)",
        "};",
        "",
        "// kFrozenCfg[path][class]: path PT_PATH_FWD/DX/DK, class light/medium/heavy.",
        "constexpr LaunchCfg kFrozenCfg[3][3] = {",
    ]
    for p, name in zip(PATHS, ("FWD", "DX", "DK")):
        cells = ", ".join("{%d, %d, %d, %d}" % tuple(policy[p][c]) for c in CLASSES)
        lines.append(f"    {{{cells}}},  // {name}: light, medium, heavy")
    lines += ["};", "",
              "// kFrozenEngine[path][class]: PT_ENGINE_FFMA (0) or PT_ENGINE_TENSOR (1); the",
              "// tensor engine only ever applies to FWD/DX at L % 4 == 0.",
              "constexpr int kFrozenEngine[3][3] = {"]
    for p, name in zip(PATHS, ("FWD", "DX", "DK")):
        cells = ", ".join(str(ENGINES.index(engines[p][c]) if engines else 0) for c in CLASSES)
        lines.append(f"    {{{cells}}},  // {name}: light, medium, heavy")
    lines += ["};", ""]
    lines += _header_backward_block(HEADER.read_text() if HEADER.exists() else None)
    lines += ["", f'constexpr const char* kFrozenCfgSource = "{source}";', "", "}  // namespace pt", ""]
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# GPU sweep
# ---------------------------------------------------------------------------
def _make_inputs(case: ShapeCase, seed: int, B: int, device):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, case.H, case.L, device=device, generator=g)
    k = torch.randn(case.H, case.K, device=device, generator=g) / (case.K ** 0.5)
    dy = torch.randn(B, case.H, case.L, device=device, generator=g)
    return x, k, dy


def _validate(case: ShapeCase, seed: int, device) -> dict[str, float]:
    """Max normalised error of each path at B<=128 against torch conv1d (TF32 off)."""
    import torch
    import torch.nn.functional as F

    from . import ops

    Bv = min(case.B, 128)
    x, k, dy = _make_inputs(case, seed, Bv, device)
    y = ops.fwd(x, k)
    gx = ops.dx(dy, k)
    gk = torch.empty_like(k)
    ops.dk(dy, x, gk)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)
    left = case.K // 2
    yr = F.conv1d(F.pad(xr, (left, case.K - 1 - left)), kr.unsqueeze(1), groups=case.H)
    gxr, gkr = torch.autograd.grad(yr, (xr, kr), dy)
    err = {}
    for name, a, b in (("fwd", y, yr), ("bwd_input", gx, gxr), ("bwd_weight", gk, gkr)):
        err[name] = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    return err


def run_sweep(cases: list[ShapeCase], warmup: int, runs: int, trial: int, seed: int, out: Path,
              reps: int = 3) -> None:
    """Time every candidate on every shape.  Within a shape the candidates are
    visited round-robin `reps` times (each visit: warm-up, then `runs` timed
    launches), and a candidate's figure is the median of its per-visit means, so
    slow drifts of the SM clock (power capping) average out instead of
    favouring whichever candidate ran first."""
    import torch

    from . import ops

    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", torch.cuda.current_device())
    out.mkdir(parents=True, exist_ok=True)
    # The candidates are launch configurations of the CUDA-core kernels: keep
    # every path on them for the sweep (the tensor engine ignores these knobs).
    for p in PATHS:
        ops.set_engine(p, "ffma")
    order = cases if trial % 2 else list(reversed(cases))
    cands = candidates() if trial % 2 else list(reversed(candidates()))
    raw_rows, summ = [], []
    stream = torch.cuda.current_stream()
    for case in order:
        sd = case_seed(seed, case)
        valid: dict[tuple, dict[str, float]] = {}
        for cand in cands:
            for p in PATHS:
                ops.set_config(p, *cand)
            valid[cand] = _validate(case, sd, dev)
        x, k, dy = _make_inputs(case, sd, case.B, dev)
        y, gx, gk = torch.empty_like(x), torch.empty_like(x), torch.empty_like(k)
        launch = {
            "fwd": lambda: ops.fwd(x, k, y),
            "bwd_input": lambda: ops.dx(dy, k, gx),
            "bwd_weight": lambda: ops.dk(dy, x, gk, mode="deterministic"),
        }
        # Candidates whose clamped launch is identical (CTAs per SM limited by
        # occupancy, stages by shared memory) are measured once: the first one
        # of each effective launch is timed and the others alias it.
        effective: dict[tuple, tuple] = {}
        alias: dict[tuple, tuple] = {}
        for cand in cands:
            for p in PATHS:
                ops.set_config(p, *cand)
            for p in PATHS:
                info = ops.kernel_info(p, case.B, case.H, case.L, case.K)
                key = (p, info["grid"], info["dynamic_smem_bytes"], info["threads_per_block"])
                alias[(cand, p)] = effective.setdefault(key, cand)
        visits: dict[tuple, list[float]] = {}
        for rep in range(reps):
            for cand in (cands if rep % 2 == 0 else list(reversed(cands))):
                for p in PATHS:
                    ops.set_config(p, *cand)
                for p in PATHS:
                    if alias[(cand, p)] != cand:
                        continue
                    if valid[cand][p] > (1e-5 if p != "bwd_weight" else 1e-4):
                        continue
                    for _ in range(warmup):
                        launch[p]()
                    ev = []
                    for _ in range(runs):
                        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        s.record(stream)
                        launch[p]()
                        e.record(stream)
                        ev.append((s, e))
                    torch.cuda.synchronize()
                    ms = [s.elapsed_time(e) for s, e in ev]
                    visits.setdefault((cand, p), []).append(statistics.mean(ms))
                    for i, v in enumerate(ms):
                        raw_rows.append({"config_id": case.config_id, "trial": trial, "rep": rep, "phase": p,
                                         "candidate": candidate_id(cand), "run": i, "runtime_ms": v})
        for cand in cands:
            for p in PATHS:
                for q in PATHS:
                    ops.set_config(q, *cand)
                base = {**asdict(case), "trial": trial, "phase": p, "rows": cand[0], "stages": cand[1],
                        "ctas_per_sm": cand[2], "threads_per_row": cand[3], "max_norm_err": valid[cand][p]}
                src = alias[(cand, p)]
                if (src, p) not in visits:
                    summ.append({**base, "valid": False})
                    continue
                v = visits[(src, p)]
                base["alias_of"] = candidate_id(src) if src != cand else ""
                info = ops.kernel_info(p, case.B, case.H, case.L, case.K)
                summ.append({**base, "valid": True, "mean_ms": statistics.median(v), "visits": len(v),
                             "visit_spread_pct": 100.0 * (max(v) / min(v) - 1.0),
                             "grid": info["grid"], "resident_blocks_per_sm": info["resident_blocks_per_sm"]})
        del x, k, dy, y, gx, gk
        torch.cuda.empty_cache()
    for p in PATHS:
        ops.set_config(p, 0)
        ops.set_engine(p, None)
    _write_csv(out / "raw.csv", raw_rows)
    _write_csv(out / "summary.csv", summ)
    (out / "metadata.json").write_text(json.dumps({
        "trial": trial, "warmup": warmup, "runs": runs, "reps": reps, "seed": seed,
        "device": torch.cuda.get_device_name(),
        "cases": [asdict(c) for c in cases], "candidates": [candidate_id(c) for c in candidates()],
        "created_unix": time.time(),
        "measurement_contract": {"strict_fp32": True, "cuda_event_kernel_timing": True,
                                 "validation_timed": False, "dk_mode": "deterministic",
                                 "candidate_order": "round-robin, direction alternating per visit; "
                                                    "reversed on even trials",
                                 "shape_order": "listed on odd trials; reversed on even trials",
                                 "figure": "median over visits of the per-visit mean",
                                 "engine": "ffma on every path (the candidates are its launch knobs)"}},
        indent=1))


def run_engine_sweep(cases: list[ShapeCase], warmup: int, runs: int, seed: int, out: Path,
                     reps: int = 3) -> list[dict]:
    """Time FWD and dX of every shape with L % 4 == 0 on both engines (FFMA at
    its frozen launch), visits alternating between engines; figure = median
    over visits of the per-visit mean."""
    import torch

    from . import ops

    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", torch.cuda.current_device())
    out.mkdir(parents=True, exist_ok=True)
    stream = torch.cuda.current_stream()
    rows = []
    try:
        for case in cases:
            if not tensor_applicable(case.L):
                continue
            sd = case_seed(seed, case)
            valid = {}
            for e in ENGINES:
                for p in ENGINE_PATHS:
                    ops.set_engine(p, e)
                valid[e] = _validate(case, sd, dev)
            x, k, dy = _make_inputs(case, sd, case.B, dev)
            y, gx = torch.empty_like(x), torch.empty_like(x)
            launch = {"fwd": lambda: ops.fwd(x, k, y), "bwd_input": lambda: ops.dx(dy, k, gx)}
            visits: dict[tuple, list[float]] = {}
            for rep in range(reps):
                for e in (ENGINES if rep % 2 == 0 else tuple(reversed(ENGINES))):
                    for p in ENGINE_PATHS:
                        ops.set_engine(p, e)
                        if valid[e][p] > 1e-5:
                            continue
                        for _ in range(warmup):
                            launch[p]()
                        ev = []
                        for _ in range(runs):
                            s, f = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            s.record(stream)
                            launch[p]()
                            f.record(stream)
                            ev.append((s, f))
                        torch.cuda.synchronize()
                        visits.setdefault((e, p), []).append(statistics.mean(s.elapsed_time(f) for s, f in ev))
            for (e, p), v in sorted(visits.items()):
                rows.append({"config_id": case.config_id, "B": case.B, "H": case.H, "L": case.L, "K": case.K,
                             "class": intensity_class(case.L, case.K), "phase": p, "engine": e,
                             "mean_ms": statistics.median(v), "visits": len(v), "max_norm_err": valid[e][p]})
            del x, k, dy, y, gx
            torch.cuda.empty_cache()
    finally:
        for p in ENGINE_PATHS:
            ops.set_engine(p, None)
    _write_csv(out / "engines.csv", rows)
    return rows


def run_backward_sweep(cases: list[ShapeCase], warmup: int, runs: int, seed: int, out: Path,
                       reps: int = 3) -> list[dict]:
    """Per shape: every distinct backward variant the candidate policies lead
    to (kernel kind and grid, as the library reports them for that policy) is
    checked against dX then dK on the same inputs and timed (per-launch CUDA
    events, visits alternating between variants; figure = median over visits of
    the per-visit mean)."""
    import torch

    from . import _lib, ops

    dev = torch.device("cuda", torch.cuda.current_device())
    out.mkdir(parents=True, exist_ok=True)
    stream = torch.cuda.current_stream()
    rows = []
    for case in cases:
        B, H, L, K = case.B, case.H, case.L, case.K
        sd = case_seed(seed, case)
        x, k, dy = _make_inputs(case, sd, B, dev)
        variants: dict[tuple, tuple] = {}
        for pol in BWD_POLICIES:
            o = _lib.LaunchOpts.frozen()
            o.bwd_kernel, o.helper_channels = pol
            kind = ops.backward_kind(B, H, L, K, opts=o)
            grid = ops.kernel_info("bwd_fused", B, H, L, K, opts=o)["grid"] if kind != "separate" else 0
            variants.setdefault((kind, grid), (o, []))[1].append(bwd_policy_id(pol))
        sep = _lib.LaunchOpts.frozen()
        sep.bwd_kernel = _lib.PT_BWD_SEPARATE
        gk0 = torch.empty_like(k)
        gx0 = ops.dx_dk(dy, x, k, gk0, opts=sep)
        gx, gk = torch.empty_like(x), torch.empty_like(k)
        err = {}
        for key, (o, _) in variants.items():
            ops.dx_dk(dy, x, k, gk, gx=gx, opts=o)
            err[key] = max(float((gx - gx0).abs().max() / gx0.abs().max().clamp_min(1e-30)),
                           float((gk - gk0).abs().max() / gk0.abs().max().clamp_min(1e-30)))
        assert ops.device_error() == 0, f"{case.config_id}: a kernel wait expired"
        keys = [kk for kk in variants if err[kk] <= 1e-4]
        visits: dict[tuple, list[float]] = {}
        for rep in range(reps):
            for key in (keys if rep % 2 == 0 else list(reversed(keys))):
                o = variants[key][0]
                for _ in range(warmup):
                    ops.dx_dk(dy, x, k, gk, gx=gx, opts=o)
                ev = []
                for _ in range(runs):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    ops.dx_dk(dy, x, k, gk, gx=gx, opts=o)
                    b.record(stream)
                    ev.append((a, b))
                torch.cuda.synchronize()
                visits.setdefault(key, []).append(statistics.mean(a.elapsed_time(b) for a, b in ev))
        for key, (o, pids) in variants.items():
            rows.append({"config_id": case.config_id, "B": B, "H": H, "L": L, "K": K,
                         "class": intensity_class(L, K), "variant": key[0], "grid": key[1],
                         "policies": ";".join(pids), "max_norm_err": err[key], "valid": err[key] <= 1e-4,
                         "mean_ms": statistics.median(visits[key]) if key in visits else float("nan"),
                         "visits": len(visits.get(key, []))})
        print(json.dumps({"config_id": case.config_id,
                          **{f"{kk[0]}@{kk[1]}": round(statistics.median(v), 4) for kk, v in visits.items()}}),
              flush=True)
        del x, k, dy, gx, gx0
        torch.cuda.empty_cache()
    _write_csv(out / "backward.csv", rows)
    return rows


def apply_engines_to_header(text: str, engines: dict[str, dict[str, str]]) -> str:
    """Rewrite only the kFrozenEngine table of an existing frozen-config header."""
    start = text.index("constexpr int kFrozenEngine[3][3] = {")
    end = text.index("};", start) + 2
    rows = ["constexpr int kFrozenEngine[3][3] = {"]
    for p, name in zip(PATHS, ("FWD", "DX", "DK")):
        cells = ", ".join(str(ENGINES.index(engines[p][c])) for c in CLASSES)
        rows.append(f"    {{{cells}}},  // {name}: light, medium, heavy")
    rows.append("};")
    return text[:start] + "\n".join(rows) + text[end:]


def _write_csv(path: Path, rows: list[dict]) -> None:
    if not rows:
        path.write_text("")
        return
    keys = list(dict.fromkeys(k for r in rows for k in r))
    with path.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=keys)
        w.writeheader()
        w.writerows(rows)


def _read_csv(path: Path) -> list[dict]:
    with path.open() as f:
        return list(csv.DictReader(f))


def aggregate_trials(root: Path) -> list[dict]:
    """Mean over trials of each (shape, phase, candidate) mean_ms; invalid rows dropped."""
    acc: dict[tuple, list[float]] = {}
    shape: dict[str, tuple[int, int]] = {}
    for t in sorted(root.glob("trial*/summary.csv")):
        for r in _read_csv(t):
            shape[r["config_id"]] = (int(r["L"]), int(r["K"]))
            if r.get("valid") != "True":
                continue
            key = (r["config_id"], r["phase"], *_cand(r))
            acc.setdefault(key, []).append(float(r["mean_ms"]))
    return [{"config_id": k[0], "phase": k[1], "rows": k[2], "stages": k[3], "ctas_per_sm": k[4],
             "threads_per_row": k[5], "L": shape[k[0]][0], "K": shape[k[0]][1],
             "mean_ms": statistics.mean(v), "trials": len(v)}
            for k, v in sorted(acc.items())]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--mode", choices=("run", "aggregate", "regret", "engines", "baselines", "backward"),
                    required=True)
    ap.add_argument("--preset", default="pathtile-train", choices=sorted(PRESETS))
    ap.add_argument("--out", type=Path, required=True, help="results directory of this preset")
    ap.add_argument("--trial", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--runs", type=int, default=20)
    ap.add_argument("--reps", type=int, default=3, help="round-robin visits per candidate and shape")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--write-header", action="store_true",
                    help="aggregate: rewrite pt_frozen_config.h; engines: rewrite its engine table")
    ap.add_argument("--per-class", action="store_true", help="aggregate: select per intensity class")
    ap.add_argument("--policy", type=Path, help="regret: frozen_config.json to score")
    ap.add_argument("--engines", type=Path, help="aggregate: engine_policy.json to include in the header")
    ap.add_argument("--bwd-policy", type=Path, help="backward: backward_policy.json to score instead of selecting")
    ap.add_argument("--train-csv", type=Path, help="baselines: candidate summary of the tuning shapes")
    ap.add_argument("--eval-csv", type=Path, help="baselines: candidate summary of the shapes to score "
                    "(default: aggregate the trials under --out)")
    args = ap.parse_args()
    if args.mode == "baselines":
        train = _read_csv(args.train_csv)
        evalset = _read_csv(args.eval_csv) if args.eval_csv else aggregate_trials(args.out)
        rows, summary = evaluate_baselines(train, evalset)
        args.out.mkdir(parents=True, exist_ok=True)
        _write_csv(args.out / "selector_baselines_per_shape.csv", rows)
        (args.out / "selector_baselines_summary.json").write_text(json.dumps(summary, indent=1))
        print(json.dumps(summary, indent=1))
        return
    if args.mode == "backward":
        rows = [r for r in run_backward_sweep(cases_for_preset(args.preset), args.warmup, args.runs, args.seed,
                                              args.out, reps=args.reps) if r["valid"]]
        if args.bwd_policy:
            pol = {c: tuple(v) for c, v in json.loads(args.bwd_policy.read_text())["policy"].items()}
        else:
            pol = select_backward(rows)
        reg = backward_regret(rows, pol)
        gains = [r["gain_vs_separate_pct"] for r in reg if r["gain_vs_separate_pct"] is not None]
        doc = {"policy": {c: list(v) for c, v in pol.items()},
               "policy_meaning": "[bwd_kernel (0 separate, 1 tensor-core fused, 2 CUDA-core fused, 3 any fused), "
                                 "most channels per helper CTA (0: none)]",
               "preset": args.preset, "selected_here": args.bwd_policy is None,
               "shapes": len(reg),
               "regret_pct_mean": statistics.mean(r["regret_pct"] for r in reg) if reg else None,
               "regret_pct_max": max(r["regret_pct"] for r in reg) if reg else None,
               "within_2pct": sum(r["regret_pct"] <= 2.0 for r in reg),
               "gain_vs_separate_pct_mean": statistics.mean(gains) if gains else None}
        _write_csv(args.out / "backward_regret.csv", reg)
        (args.out / ("backward_policy.json" if args.bwd_policy is None else "backward_scored.json")).write_text(
            json.dumps(doc, indent=1))
        print(json.dumps(doc, indent=1))
        if args.write_header and args.bwd_policy is None:
            HEADER.write_text(apply_backward_to_header(HEADER.read_text(), pol))
        return
    if args.mode == "engines":
        rows = run_engine_sweep(cases_for_preset(args.preset), args.warmup, args.runs, args.seed, args.out,
                                reps=args.reps)
        engines = select_engines(rows)
        reg = engine_regret(rows, engines)
        doc = {"engines": engines, "tuning_preset": args.preset,
               "shapes": sorted({r["config_id"] for r in rows}),
               "regret_pct_mean": statistics.mean(r["regret_pct"] for r in reg) if reg else None,
               "gain_vs_ffma_pct_mean": statistics.mean(r["gain_vs_ffma_pct"] for r in reg) if reg else None}
        _write_csv(args.out / "engine_regret.csv", reg)
        (args.out / "engine_policy.json").write_text(json.dumps(doc, indent=1))
        print(json.dumps(doc, indent=1))
        if args.write_header:
            HEADER.write_text(apply_engines_to_header(HEADER.read_text(), engines))
    elif args.mode == "run":
        run_sweep(cases_for_preset(args.preset), args.warmup, args.runs, args.trial, args.seed,
                  args.out / f"trial{args.trial}", reps=args.reps)
    elif args.mode == "aggregate":
        summary = aggregate_trials(args.out)
        policy = select_policy(summary, per_class=args.per_class)
        _write_csv(args.out / "aggregate_summary.csv", summary)
        reg = regret_table(summary, policy)
        doc = {"policy": {p: {c: dict(zip(("rows", "stages", "ctas_per_sm", "threads_per_row"), policy[p][c]))
                              for c in CLASSES}
                          for p in PATHS},
               "per_class": args.per_class,
               "tuning_preset": args.preset, "tuning_shapes": sorted({r["config_id"] for r in summary}),
               "training_regret_pct_mean": statistics.mean(r["regret_pct"] for r in reg)}
        (args.out / "frozen_config.json").write_text(json.dumps(doc, indent=1))
        print(json.dumps(doc, indent=1))
        if args.write_header:
            engines = json.loads(args.engines.read_text())["engines"] if args.engines else None
            HEADER.write_text(render_header(policy, f"B200 sweep of preset {args.preset}", engines))
    else:
        summary = aggregate_trials(args.out)
        pol = json.loads(args.policy.read_text())["policy"]
        policy = {p: {c: (pol[p][c]["rows"], pol[p][c]["stages"], pol[p][c]["ctas_per_sm"],
                          pol[p][c].get("threads_per_row", 1)) for c in CLASSES}
                  for p in PATHS}
        reg = regret_table(summary, policy)
        _write_csv(args.out / "regret.csv", reg)
        vals = [r["regret_pct"] for r in reg]
        print(json.dumps({"shapes": len(vals), "mean_regret_pct": statistics.mean(vals),
                          "max_regret_pct": max(vals),
                          "within_1pct": sum(v <= 1.0 for v in vals),
                          "within_2pct": sum(v <= 2.0 for v in vals)}, indent=1))


if __name__ == "__main__":
    main()
