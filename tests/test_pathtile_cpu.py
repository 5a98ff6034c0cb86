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
                    "ctas_per_sm": cand[2], "mean_ms": ms})
    return out


def test_select_policy_sums_over_shapes_and_breaks_ties_low():
    a, b, c = (64, 2, 1), (128, 3, 2), (256, 2, 1)
    table = []
    for phase in pt.PATHS:
        table += [("s1", phase, a, 1.0), ("s1", phase, b, 0.5), ("s1", phase, c, 0.9),
                  ("s2", phase, a, 1.0), ("s2", phase, b, 2.0), ("s2", phase, c, 0.6)]
    pol = pt.select_policy(_rows(table))
    # sums: a=2.0, b=2.5, c=1.5 -> c for every path, although b wins s1.
    assert all(pol[p] == c for p in pt.PATHS)
    tie = _rows([("s1", p, a, 1.0) for p in pt.PATHS] + [("s1", p, c, 1.0) for p in pt.PATHS])
    assert all(v == a for v in pt.select_policy(tie).values())


def test_candidate_missing_a_shape_is_not_eligible():
    a, b = (64, 2, 1), (128, 3, 2)
    rows = []
    for p in pt.PATHS:
        rows += [("s1", p, a, 5.0), ("s2", p, a, 5.0), ("s1", p, b, 0.1)]  # b failed on s2
    assert all(v == a for v in pt.select_policy(_rows(rows)).values())


def test_regret_against_per_shape_oracle():
    a, b = (64, 2, 1), (128, 3, 2)
    rows = []
    for p in pt.PATHS:
        rows += [("s1", p, a, 1.0), ("s1", p, b, 0.8), ("s2", p, a, 1.0), ("s2", p, b, 1.25)]
    pol = {p: a for p in pt.PATHS}
    reg = {r["config_id"]: r["regret_pct"] for r in pt.regret_table(_rows(rows), pol)}
    assert reg["s1"] == pytest.approx(25.0)
    assert reg["s2"] == pytest.approx(0.0)


def test_render_header_is_parseable_table():
    pol = {"fwd": (128, 3, 2), "bwd_input": (64, 4, 3), "bwd_weight": (256, 2, 1)}
    text = pt.render_header(pol, "unit test")
    entries = re.findall(r"\{(\d+), (\d+), (\d+)\},\s+// (FWD|DX|DK)", text)
    assert entries == [("128", "3", "2", "FWD"), ("64", "4", "3", "DX"), ("256", "2", "1", "DK")]
    assert 'kFrozenCfgSource = "unit test"' in text


def test_committed_header_matches_renderer_layout():
    text = pt.HEADER.read_text()
    assert len(re.findall(r"\{(\d+), (\d+), (\d+)\},\s+// (FWD|DX|DK)", text)) == 3


def test_case_seed_rule():
    c = pt.PATHTILE_TRAIN_CASES[0]
    import zlib

    assert pt.case_seed(42, c) == 42 + zlib.crc32(c.config_id.encode())
