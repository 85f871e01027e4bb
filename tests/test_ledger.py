"""Measurements as ledger facts (the analysis ledger as the
measurement store; reference pdum/tl/analysis.py:121-175 and
conformance/test_fusion_triton.py:87-117).  The device timing is replaced by a
counter here; the GPU test measures for real."""

import json

import pytest


def _flash_plan():
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    return plan_region(flash_tile(T=256, E=64, OD=64, SI=2).naive)


def test_a_keyed_measurement_is_taken_once(dsl, monkeypatch, tmp_path):
    from pdum.tl.analysis import no_reanalysis, save_ledger

    from pdum_dsl_b200 import ledger

    calls = []
    monkeypatch.setattr(ledger, "_time_us", lambda kernel, dtype, reps: calls.append(dtype) or 12.5)
    (g,) = _flash_plan().groups
    fact = ledger.sm100_us(g.kernel, machine="cpu-test-fake", dtype="bf16", reps=3)
    assert fact.value == {"us": 12.5, "reps": 3, "dtype": "bf16", "machine": "cpu-test-fake"}
    with no_reanalysis():  # the warmth law: a keyed measurement is never repeated
        again = ledger.sm100_us(g.kernel, machine="cpu-test-fake", dtype="bf16", reps=3)
    assert again.key == fact.key and calls == ["bf16"]
    other = ledger.sm100_us(g.kernel, machine="cpu-test-fake", dtype="f32", reps=3)
    assert other.key != fact.key and calls == ["bf16", "f32"]
    prof = ledger.sm100_profile(g.kernel, {"dram_bytes": 1.0e6, "tensor_active_pct": 51.1}, machine="cpu-test-fake")
    assert prof.value["tensor_active_pct"] == 51.1
    path = tmp_path / "ledger.json"
    assert save_ledger(path) >= 3
    saved = json.loads(path.read_text())
    assert {rec["analysis"] for rec in saved.values()} >= {"fusion.sm100a-us@v1", "fusion.sm100a-profile@v1"}


def test_measured_groups_turn_green(dsl, monkeypatch):
    from pdum_dsl_b200 import ledger

    monkeypatch.setattr(ledger, "_time_us", lambda kernel, dtype, reps: 7.0)
    plan = _flash_plan()
    green, facts = ledger.green_plan(plan, machine="cpu-test-fake-2", reps=2)
    assert [g.confidence for g in green.groups] == ["green"]
    assert facts[0].value["us"] == 7.0
    assert plan.groups[0].confidence != "green"  # the input plan is unchanged


def test_profile_facts_must_be_plain_data(dsl):
    from pdum_dsl_b200 import ledger

    (g,) = _flash_plan().groups
    with pytest.raises(TypeError):
        ledger.sm100_profile(g.kernel, {"bad": object()}, machine="cpu-test-fake-3")
