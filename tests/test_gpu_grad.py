"""The autodiff joint of attention lowered whole: compile_grad(RegionGrad) vs run_region."""

import numpy as np
import pytest

from tests.golden import load
from tests.tolerances import assert_bf16

pytestmark = pytest.mark.gpu


def _joint(region):
    from pdum.tl.autodiff import grad

    out = region.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(region.params)}
    names[id(out)] = "out"
    return grad(region, "out", seed="dO", names=names)


def test_flash_tile_joint_matches_the_reference_evaluation(cuda, dsl):
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.grad import compile_grad

    spec, ins, outs = load("flash_joint_bwd_d64")
    rg = _joint(flash_tile(T=200, E=64, OD=64, SI=2).naive)
    got = compile_grad(rg)(ins)
    assert len(got) == 4
    assert_bf16(got[0], outs[0], what="out")
    qs = spec["inputs"][0]["scale"]  # bf16 bar on the gradient w.r.t. the unit-variance query
    assert_bf16(got[1] * qs, outs[1] * qs, what="dq")
    assert_bf16(got[2], outs[2], what="dk")
    assert_bf16(got[3], outs[3], what="dv (o, s)")


def test_scaled_rider_gqa_joint_vs_run_region(cuda, dsl):
    from pdum.tl.dialect import run_region
    from pdum.tl.tensor import Tensor

    from pdum_dsl_b200.grad import compile_grad
    from pdum_dsl_b200.regions import attention_region
    from tests.golden import round_bf16

    rg = _joint(attention_region(B=1, H=2, T=130, D=64, causal=True, scale=0.125, group=2))
    rng = np.random.default_rng(3)
    vals, arrs = [], []
    for p in rg.region.params:
        dims = p.type.dims
        a = round_bf16(rng.standard_normal(tuple(d.stop - d.start for d in dims)))
        arrs.append(a)
        vals.append(Tensor.from_numpy(a, tuple(d.name for d in dims)))
    want = run_region(rg.region, vals)
    got = compile_grad(rg)(arrs)
    for g, w in zip(got, want):
        assert_bf16(g, w.to_numpy(order=w.names))


def test_model_plan_executes_carve_by_carve(cuda, dsl):
    """The carved backward plan run carve by carve, device carves on the sm_100a library
    (f32 IEEE column) and the rest through run_region, reproduces run_region of the
    whole joint."""
    from pdum.tl.dialect import run_region
    from pdum.tl.partition import plan_model
    from pdum.tl.tensor import Tensor
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.plan import execute_model_plan
    from tests.tolerances import assert_f32

    rg = _joint(flash_tile(T=64, E=8, OD=8, SI=2).naive)
    plan = plan_model(rg.region)
    rng = np.random.default_rng(5)
    ins = []
    for p in rg.region.params:
        dims = p.type.dims
        ins.append(Tensor.from_numpy(rng.standard_normal(tuple(d.stop - d.start for d in dims)),
                                     tuple(d.name for d in dims)))
    want = run_region(rg.region, list(ins))
    got, assign = execute_model_plan(plan, rg.region, ins)
    assert assign.count("device") >= 3
    for g, w in zip(got, want):
        assert_f32(g.to_numpy(order=w.names), w.to_numpy(order=w.names))
