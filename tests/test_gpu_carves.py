"""The carved attention backward (plan_model of the autodiff joint) run carve by
carve on the device, every carve on the sm_100a library, against the reference's
own evaluation (run_region) of the joint and of each carve."""

import numpy as np
import pytest

from tests.tolerances import assert_f32

pytestmark = pytest.mark.gpu


def _joint(region):
    from pdum.tl.autodiff import grad

    out = region.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(region.params)}
    names[id(out)] = "out"
    return grad(region, "out", seed="dO", names=names)


def _inputs(region, seed, scale_first=1.0):
    from pdum.tl.tensor import Tensor

    rng = np.random.default_rng(seed)
    arrs, tens = [], []
    for i, p in enumerate(region.params):
        dims = p.type.dims
        a = rng.standard_normal(tuple(d.stop - d.start for d in dims))
        arrs.append(a)
        tens.append(Tensor.from_numpy(a, tuple(d.name for d in dims)))
    return arrs, tens


@pytest.mark.parametrize("T,E,OD", [(64, 8, 8), (200, 64, 64), (130, 32, 48)])
def test_joint_carve_by_carve_all_on_device(cuda, dsl, T, E, OD):
    import torch
    from pdum.tl.dialect import run_region
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.plan import device_assignment, execute_model_plan

    rg = _joint(flash_tile(T=T, E=E, OD=OD, SI=2).naive)
    plan = plan_model(rg.region)
    carves = [c for c in plan.carves if c.root is not None]
    assert device_assignment(plan) == ["device"] * len(carves)
    arrs, tens = _inputs(rg.region, 5)
    want = run_region(rg.region, list(tens))
    got, assign = execute_model_plan(plan, rg.region, [torch.tensor(a, dtype=torch.float32, device=cuda)
                                                       for a in arrs])
    assert assign == ["device"] * len(carves)
    for g, w, what in zip(got, want, ("out", "dq", "dk", "dv")):
        assert_f32(g.cpu().numpy(), w.to_numpy(order=w.names), what=what)


def _reference_carve_values(plan, region, tens):
    """The reference's own carve-by-carve execution (run_region per carve, as
    packages/tensorlib/tests/test_partition.py:124-193 runs it) -> per carve its
    input Tensors and outputs.  Test-side checker only."""
    from pdum.tl.dialect import run_region

    from pdum_dsl_b200.plan import _CHART_OPS, _bare

    vals = {id(p): v for p, v in zip(region.params, tens)}

    def known(b):
        while id(b) not in vals and b.op in _CHART_OPS:
            b = b.args[0]
        return b

    per = {}
    pending = [(i, c) for i, c in enumerate(plan.carves) if c.root is not None]
    while pending:
        for i, c in list(pending):
            bounds = [known(b) for b in c.bounds]
            if not all(id(b) in vals for b in bounds):
                continue
            ins = [vals[id(b)] for b in bounds]
            got = run_region(c.kernel, ins)
            outs = tuple(got) if isinstance(got, (tuple, list)) else (got,)
            for node, val in zip((c.root, *c.artifacts), outs):
                vals[id(node)] = val
                vals[id(_bare(node))] = val
            per[i] = (ins, outs)
            pending.remove((i, c))
    return per


def _widened_joint(kind):
    from pdum_dsl_b200.regions import attention_region

    kw = {"riders": dict(B=2, H=2, T=40, D=16, causal=True, scale=0.3),
          "gqa": dict(B=1, H=2, T=33, D=16, causal=True, scale=0.3, group=2),
          "window": dict(T=72, D=16, causal=True, window=20, scale=0.3),
          "block": dict(T=72, D=16, causal=False, block=24, scale=0.3)}[kind]
    return _joint(attention_region(**kw))


@pytest.mark.parametrize("kind", ["riders", "gqa", "window", "block"])
def test_widened_joints_carve_by_carve_all_on_device(cuda, dsl, kind):
    """Joints of widened regions (batch / head riders, a GQA group, sliding-window and
    block-diagonal masks): plan_model carves them differently (rider carves are rank 3-5),
    and every carve still runs on the device, matching run_region of the joint."""
    import torch
    from pdum.tl.dialect import run_region
    from pdum.tl.partition import plan_model

    from pdum_dsl_b200.plan import device_assignment, execute_model_plan

    rg = _widened_joint(kind)
    plan = plan_model(rg.region)
    n = sum(c.root is not None for c in plan.carves)
    assert device_assignment(plan) == ["device"] * n
    arrs, tens = _inputs(rg.region, 6)
    want = run_region(rg.region, list(tens))
    got, _ = execute_model_plan(plan, rg.region, [torch.tensor(a, dtype=torch.float32, device=cuda) for a in arrs])
    for g, w, what in zip(got, want, ("out", "dq", "dk", "dv")):
        assert_f32(g.cpu().numpy(), w.to_numpy(order=w.names), what=f"{kind} {what}")


@pytest.mark.parametrize("T,E", [(96, 16), (160, 64)])
def test_each_carve_matches_run_region_on_the_reference_boundary_values(cuda, dsl, T, E):
    """Every carve alone (score-space programs, the flash carve and the GEMM carves),
    fed the boundary values the reference's own carve-by-carve run produces, against
    run_region of that carve."""
    import torch
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.plan import _lowered
    from pdum_dsl_b200.score_program import ScoreProgramSpec

    rg = _joint(flash_tile(T=T, E=E, OD=E, SI=2).naive)
    plan = plan_model(rg.region)
    _, tens = _inputs(rg.region, 11)
    per = _reference_carve_values(plan, rg.region, tens)
    n_sp = 0
    for i, c in enumerate(plan.carves):
        if c.root is None:
            continue
        run, kernel = _lowered(c)
        n_sp += isinstance(run.spec, ScoreProgramSpec)
        ins, outs = per[i]
        dev = [torch.tensor(t.to_numpy(order=tuple(d.name for d in p.type.dims)), dtype=torch.float32,
                            device=cuda) for t, p in zip(ins, kernel.params)]
        got = run.run_t(*dev)
        got = got if isinstance(got, tuple) else (got,)
        for g, w in zip(got, outs):
            w = w.to_numpy(order=w.names)
            g = g.float().cpu().numpy()
            if np.abs(w).max() < 1e-8:  # the m gradient: exactly zero in exact arithmetic
                assert np.abs(g).max() < 1e-4, c.root_op
            else:
                assert_f32(g, w, what=f"carve {i} {c.group.template}")
    assert n_sp >= 4
