"""CPU tests of the PathTile offline selection: presets, the argmin-of-summed-
latency policy with its tie rule, regret, and the frozen header it writes."""
from __future__ import annotations

import re

import pytest

from pathtile_b200 import pathtile as pt


def test_presets_match_reference_and_spec():
    train = pt.cases_for_preset("pathtile-train")
    hold = pt.cases_for_preset("pathtile-holdout")
    sweep = pt.cases_for_preset("heldout-sweep")
    assert len(train) == 20 and len(hold) == 10
    assert len(sweep) == 81
    assert train[0] == pt.ShapeCase("main_b16384_h128_l48_k48", 16384, 128, 48, 48, "main")
    assert {(c.L, c.K) for c in sweep} == set(pt.SWEEP_LK)
    assert all(c.K <= c.L for c in sweep)
    assert len({c.config_id for c in train + hold + sweep}) == 111


def test_invalid_case_rejected():
    with pytest.raises(ValueError):
        pt.ShapeCase("bad", 4, 4, 49, 3, "x").validate()
    with pytest.raises(ValueError):
        pt.cases_for_preset("nope")


def _rows(table):
    out = []
    for cid, phase, cand, ms in table:
        out.append({"config_id": cid, "phase": phase, "rows": cand[0], "stages": cand[1],
                    "ctas_per_sm": cand[2], "threads_per_row": cand[3], "mean_ms": ms})
    return out


def test_select_policy_sums_over_shapes_and_breaks_ties_low():
    a, b, c = (64, 2, 1, 1), (128, 3, 2, 1), (256, 2, 1, 2)
    table = []
    for phase in pt.PATHS:
        table += [("s1", phase, a, 1.0), ("s1", phase, b, 0.5), ("s1", phase, c, 0.9),
                  ("s2", phase, a, 1.0), ("s2", phase, b, 2.0), ("s2", phase, c, 0.6)]
    pol = pt.select_policy(_rows(table))
    # sums: a=2.0, b=2.5, c=1.5 -> c for every path and class, although b wins s1.
    assert all(pol[p][cls] == c for p in pt.PATHS for cls in pt.CLASSES)
    tie = _rows([("s1", p, a, 1.0) for p in pt.PATHS] + [("s1", p, c, 1.0) for p in pt.PATHS])
    assert all(v[cls] == a for v in pt.select_policy(tie).values() for cls in pt.CLASSES)


def test_per_class_policy_and_inheritance():
    a, b = (64, 2, 1, 1), (128, 3, 2, 2)
    rows = []
    for p in pt.PATHS:  # s_light is (24, 8) = light, s_heavy is (48, 48) = heavy
        rows += [("s_light", p, a, 1.0), ("s_light", p, b, 2.0), ("s_heavy", p, a, 3.0), ("s_heavy", p, b, 1.0)]
    shapes = {"s_light": (24, 8), "s_heavy": (48, 48)}
    table = _rows(rows)
    for r in table:
        r["L"], r["K"] = shapes[r["config_id"]]
    pol = pt.select_policy(table, per_class=True)
    for p in pt.PATHS:
        assert pol[p]["light"] == a and pol[p]["heavy"] == b
        assert pol[p]["medium"] == b  # no medium shapes: inherits (heavy before light)
    glob = pt.select_policy(table)
    assert all(glob[p][c] == b for p in pt.PATHS for c in pt.CLASSES)  # sums a=4, b=3


def test_intensity_classes():
    assert pt.intensity_class(48, 48) == "heavy"
    assert pt.intensity_class(32, 32) == "heavy"
    assert pt.intensity_class(48, 24) == "medium"
    assert pt.intensity_class(16, 16) == "medium"
    assert pt.intensity_class(24, 8) == "light"
    assert pt.intensity_class(37, 13) == "light"
    assert pt.in_range_pairs(48, 48) == 1728


def test_candidate_missing_a_shape_is_not_eligible():
    a, b = (64, 2, 1, 1), (128, 3, 2, 2)
    rows = []
    for p in pt.PATHS:
        rows += [("s1", p, a, 5.0), ("s2", p, a, 5.0), ("s1", p, b, 0.1)]  # b failed on s2
    assert all(v[c] == a for v in pt.select_policy(_rows(rows)).values() for c in pt.CLASSES)


def test_regret_against_per_shape_oracle():
    a, b = (64, 2, 1, 1), (128, 3, 2, 2)
    rows = []
    for p in pt.PATHS:
        rows += [("s1", p, a, 1.0), ("s1", p, b, 0.8), ("s2", p, a, 1.0), ("s2", p, b, 1.25)]
    table = _rows(rows)
    for r in table:
        r["L"], r["K"] = 48, 48
    pol = {p: {c: a for c in pt.CLASSES} for p in pt.PATHS}
    reg = {r["config_id"]: r["regret_pct"] for r in pt.regret_table(table, pol)}
    assert reg["s1"] == pytest.approx(25.0)
    assert reg["s2"] == pytest.approx(0.0)


HEADER_ROW = (r"\{(\{\d+, \d+, \d+, \d+\}), (\{\d+, \d+, \d+, \d+\}), (\{\d+, \d+, \d+, \d+\})\},"
              r"\s+// (FWD|DX|DK)")


def test_render_header_is_parseable_table():
    pol = {"fwd": {"light": (64, 4, 3, 2), "medium": (128, 3, 2, 1), "heavy": (128, 2, 3, 1)},
           "bwd_input": {c: (64, 4, 3, 1) for c in pt.CLASSES},
           "bwd_weight": {c: (256, 2, 1, 1) for c in pt.CLASSES}}
    text = pt.render_header(pol, "unit test")
    entries = re.findall(HEADER_ROW, text)
    assert entries[0] == ("{64, 4, 3, 2}", "{128, 3, 2, 1}", "{128, 2, 3, 1}", "FWD")
    assert [e[3] for e in entries] == ["FWD", "DX", "DK"]
    assert 'kFrozenCfgSource = "unit test"' in text


def test_committed_header_matches_renderer_layout():
    assert len(re.findall(HEADER_ROW, pt.HEADER.read_text())) == 3


def test_case_seed_rule():
    c = pt.PATHTILE_TRAIN_CASES[0]
    import zlib

    assert pt.case_seed(42, c) == 42 + zlib.crc32(c.config_id.encode())


def _erow(cid, L, K, phase, engine, ms):
    return {"config_id": cid, "L": L, "K": K, "phase": phase, "engine": engine, "mean_ms": ms}


def test_select_engines_per_class_on_summed_latency():
    rows = []
    # heavy shapes (L = K = 48): tensor faster in total although slower on h2
    for cid, f, t in (("h1", 1.0, 0.8), ("h2", 1.0, 1.1)):
        for p in pt.ENGINE_PATHS:
            rows += [_erow(cid, 48, 48, p, "ffma", f), _erow(cid, 48, 48, p, "tensor", t)]
    # light shape (K = 3): FFMA faster
    for p in pt.ENGINE_PATHS:
        rows += [_erow("l1", 48, 3, p, "ffma", 0.5), _erow("l1", 48, 3, p, "tensor", 0.6)]
    eng = pt.select_engines(rows)
    assert eng["fwd"]["heavy"] == "tensor" and eng["bwd_input"]["heavy"] == "tensor"
    assert eng["fwd"]["light"] == "ffma"
    assert eng["fwd"]["medium"] == "ffma"  # no shapes: stays on the CUDA-core kernels
    assert all(v == "ffma" for v in eng["bwd_weight"].values())
    reg = {r["config_id"]: r for r in pt.engine_regret(rows, eng)}
    assert reg["h2"]["regret_pct"] == pytest.approx(10.0)
    assert reg["h1"]["regret_pct"] == pytest.approx(0.0)
    assert reg["h1"]["gain_vs_ffma_pct"] == pytest.approx(25.0)


def test_select_engines_tie_keeps_ffma():
    rows = [_erow("s", 32, 32, p, e, 1.0) for p in pt.ENGINE_PATHS for e in pt.ENGINES]
    assert pt.select_engines(rows)["fwd"]["heavy"] == "ffma"


def test_tensor_engine_applicability():
    assert pt.tensor_applicable(48) and pt.tensor_applicable(4)
    assert not pt.tensor_applicable(37) and not pt.tensor_applicable(2)


ENGINE_ROW = r"\{(\d), (\d), (\d)\},\s+// (FWD|DX|DK)"


def test_render_header_engine_table():
    pol = {p: {c: (128, 3, 2, 1) for c in pt.CLASSES} for p in pt.PATHS}
    eng = {p: {c: "ffma" for c in pt.CLASSES} for p in pt.PATHS}
    eng["fwd"]["heavy"] = "tensor"
    eng["bwd_input"]["medium"] = "tensor"
    rows = re.findall(ENGINE_ROW, pt.render_header(pol, "t", eng))
    assert rows == [("0", "0", "1", "FWD"), ("0", "1", "0", "DX"), ("0", "0", "0", "DK")]
    assert re.findall(ENGINE_ROW, pt.render_header(pol, "t"))[0][:3] == ("0", "0", "0")
    assert len(re.findall(ENGINE_ROW, pt.HEADER.read_text())) == 3


def test_apply_engines_rewrites_only_the_engine_table():
    text = pt.HEADER.read_text()
    eng = {p: {c: "ffma" for c in pt.CLASSES} for p in pt.PATHS}
    eng["fwd"]["light"] = eng["bwd_input"]["heavy"] = "tensor"
    out = pt.apply_engines_to_header(text, eng)
    assert re.findall(ENGINE_ROW, out) == [("1", "0", "0", "FWD"), ("0", "0", "1", "DX"), ("0", "0", "0", "DK")]
    assert re.findall(HEADER_ROW, out) == re.findall(HEADER_ROW, text)
    assert out.count("constexpr int kFrozenEngine") == 1


def test_tensor_applicable_means_full_tiles():
    assert [L for L in range(1, 49) if pt.tensor_applicable(L)] == [4, 8, 12, 16, 24, 48]


def _cand_rows(cid, phase, times):
    """Summary rows of one (shape, phase): {candidate tuple: mean_ms}."""
    return [{"config_id": cid, "phase": phase, "rows": c[0], "stages": c[1], "ctas_per_sm": c[2],
             "threads_per_row": c[3], "L": 48, "K": 48, "mean_ms": v} for c, v in times.items()]


def test_selector_baselines_against_hand_computed_regret():
    A, B2, C = (128, 3, 2, 1), (128, 2, 2, 1), (256, 3, 1, 1)
    train = []
    # Candidate A wins two shapes by a hair, C wins one by a lot: the global
    # (sum) rule picks C, the majority-winner rule picks A.
    for cid, ta, tc in (("s1", 1.0, 1.01), ("s2", 1.0, 1.01), ("s3", 3.0, 1.0)):
        for ph in pt.PATHS:
            train += _cand_rows(cid, ph, {A: ta, B2: 5.0, C: tc})
    assert pt.majority_winner_policy(train) == {p: A for p in pt.PATHS}
    evalset = []
    for ph in pt.PATHS:
        evalset += _cand_rows("e1", ph, {A: 2.0, B2: 4.0, C: 1.0})
    rows, summary = pt.evaluate_baselines(train, evalset)
    assert len(rows) == 1
    r = rows[0]
    assert r["oracle_total_ms"] == pytest.approx(3.0)
    assert r["global_regret_pct"] == pytest.approx(0.0)
    assert r["majority_winner_regret_pct"] == pytest.approx(100.0)
    # default policy: FWD/dX A (2.0 each), dK B2 (4.0) -> 8.0 / 3.0
    assert r["default_regret_pct"] == pytest.approx(100.0 * (8.0 / 3.0 - 1.0))
    # random fixed: mean over the three candidates per path = 7/3, times three paths
    assert r["random_fixed_regret_pct"] == pytest.approx(100.0 * (7.0 / 3.0 - 1.0))
    assert summary["global"]["shapes"] == 1 and summary["global"]["within_2pct"] == 1


def test_host_cpu_mask_and_numa_binding_restore(monkeypatch):
    """near_device binds the calling thread to the GPU-local CPUs NVML reports
    (here a fake answer) and restores the previous affinity afterwards; with no
    answer it leaves the affinity alone."""
    import os

    from pathtile_b200 import host

    assert host.cpus_from_mask([0b1011, 1]) == [0, 1, 3, 64]
    assert host.cpus_from_mask([0]) == []
    before = os.sched_getaffinity(0)
    subset = sorted(before)[:1]
    monkeypatch.setattr(host, "device_local_cpus", lambda dev: subset + [10_000])
    with host.near_device(0) as cpus:
        assert cpus == subset
        assert os.sched_getaffinity(0) == set(subset)
    assert os.sched_getaffinity(0) == before
    monkeypatch.setattr(host, "device_local_cpus", lambda dev: [])
    with host.near_device(0) as cpus:
        assert cpus == [] and os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before


# ---------------- backward-kernel axis ----------------
def _bwd_row(cid, L, K, variant, policies, ms):
    return {"config_id": cid, "L": L, "K": K, "variant": variant, "policies": ";".join(policies), "mean_ms": ms}


def test_backward_policy_selection_and_regret():
    from pathtile_b200 import pathtile as pt

    sep, tf0, tf4, ff = "k0h0", "k1h0", "k1h4", "k2h0"
    any0, any4 = "k3h0", "k3h4"
    rows = [
        # heavy shape A: tensor fused best with helpers
        _bwd_row("A", 48, 48, "separate", [sep, ff], 3.0),
        _bwd_row("A", 48, 48, "tensor_fused", [tf0, any0], 2.0),
        _bwd_row("A", 48, 48, "tensor_fused", ["k1h2", tf4, "k1h8", "k3h2", any4, "k3h8"], 1.5),
        # heavy shape B: helpers slower
        _bwd_row("B", 48, 48, "separate", [sep, ff], 3.0),
        _bwd_row("B", 48, 48, "tensor_fused", [tf0, any0, "k1h2", "k3h2"], 2.0),
        _bwd_row("B", 48, 48, "tensor_fused", [tf4, "k1h8", any4, "k3h8"], 2.2),
        # light shape: only the CUDA-core fused kernel or separate
        _bwd_row("C", 16, 4, "separate", [sep, tf0, "k1h2", tf4, "k1h8"], 1.0),
        _bwd_row("C", 16, 4, "ffma_fused", [ff, any0, "k3h2", any4, "k3h8"], 0.7),
    ]
    pol = pt.select_backward(rows)
    # heavy: totals k1h2/k3h2 = 1.5 + 2.0 = 3.5 (the smallest; ties -> smaller tuple k1h2)
    assert pol["heavy"] == (1, 2)
    # light: any-fused policies 0.7; the smallest tuple among them is (2, 0)
    assert pol["light"] == (2, 0)
    assert pol["medium"] == pol["heavy"]  # no medium shape: inherits
    reg = {r["config_id"]: r for r in pt.backward_regret(rows, pol)}
    assert reg["A"]["regret_pct"] == 0.0 and reg["B"]["regret_pct"] == 0.0
    assert abs(reg["C"]["gain_vs_separate_pct"] - 100 * (1.0 / 0.7 - 1)) < 1e-9


def test_backward_header_rewrite_keeps_the_rest():
    from pathtile_b200 import pathtile as pt

    text = pt.HEADER.read_text()
    new = pt.apply_backward_to_header(text, {"light": (2, 0), "medium": (3, 4), "heavy": (1, 0)})
    assert "    {2, 0},  // light" in new and "    {1, 0},  // heavy" in new
    assert new.replace("{2, 0},  // light", "").count("kFrozenCfg[3][3]") == text.count("kFrozenCfg[3][3]")
    # The full header renderer keeps the backward table of the existing header.
    assert "kFrozenBwd" in pt.render_header({p: {c: (128, 3, 2, 1) for c in pt.CLASSES} for p in pt.PATHS}, "x")
