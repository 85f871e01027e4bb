"""Host logic of the score-space program family (CPU): the carves of the autodiff
joint of attention compile, with the shapes and refusals expected."""

import pytest

from pdum_dsl_b200.recognize import Untranslatable


def _joint(region):
    from pdum.tl.autodiff import grad

    out = region.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(region.params)}
    names[id(out)] = "out"
    return grad(region, "out", seed="dO", names=names)


def test_every_carve_of_the_flash_joint_lowers(dsl):
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.plan import device_assignment

    plan = plan_model(_joint(flash_tile(T=64, E=8, OD=8, SI=2).naive).region)
    assign = device_assignment(plan)
    assert assign == ["device"] * len(plan.carves), assign
    assert any(c.group.confidence == "red" for c in plan.carves)  # the max-adjoint scan is among them


@pytest.mark.parametrize("kw", [dict(B=2, H=2, T=16, D=8, causal=True, scale=0.3),
                                dict(B=1, H=2, T=16, D=8, causal=True, scale=0.3, group=2),
                                dict(T=16, D=8, causal=True, window=5), dict(T=16, D=8, causal=False, block=4)])
def test_every_carve_of_widened_joints_lowers(dsl, kw):
    """Rider joints carve into rank-3..5 pieces (map chains, red scans, contractions with
    riders); block masks bring floor / div into the carves: all lower."""
    from pdum.tl.partition import plan_model

    from pdum_dsl_b200.plan import device_assignment
    from pdum_dsl_b200.regions import attention_region

    plan = plan_model(_joint(attention_region(**kw)).region)
    assert device_assignment(plan) == ["device"] * len(plan.carves)


def test_score_program_shapes(dsl):
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.score_program import match_score_program

    plan = plan_model(_joint(flash_tile(T=64, E=8, OD=8, SI=2).naive).region)
    modes = []
    for c in plan.carves:
        try:
            sp = match_score_program(c.kernel)
        except Untranslatable:
            continue
        modes.append(tuple(p.mode for p in sp.passes))
        for p in sp.passes:
            assert p.n_regs <= 12 and len(p.ops) <= 64
    # den-grad and D-like row statistics, dV^T as a contraction over t, the scan as pre-pass + tile, dS tile
    assert ("row_sum",) in modes and ("row_contract",) in modes and ("row_min", "tile") in modes
    assert ("tile",) in modes


def test_refuses_non_score_programs(dsl):
    from pdum_dsl_b200.regions import layernorm_region
    from pdum_dsl_b200.score_program import match_score_program

    with pytest.raises(Untranslatable):
        match_score_program(layernorm_region(4, 7, eps=1e-5))
