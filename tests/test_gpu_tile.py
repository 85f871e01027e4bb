"""The drop-in boundary on silicon: reference regions -> plan_region -> compile_tile -> run.

Mirrors the reference's device tests (conformance/test_fusion_triton.py:69-346,
conformance/test_triton_tile.py:27-35), with this backend's compile_tile in
place of the Triton translator; the checker is the reference's run_region.
"""

import numpy as np
import pytest

from tests.golden import load
from tests.tolerances import assert_bf16, assert_f32

pytestmark = pytest.mark.gpu


def _tensors(region, rng):
    from pdum.tl.tensor import Tensor

    vals = []
    for p in region.params:
        dims = p.type.dims
        arr = rng.standard_normal(tuple(d.stop - d.start for d in dims))
        vals.append(Tensor.from_numpy(arr, tuple(d.name for d in dims)))
    return vals


def test_the_fused_flash_composition_runs(cuda, dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.tile import compile_tile

    f = flash_tile()
    (g,) = plan_region(f.naive).groups
    assert g.template == "flash"
    run = compile_tile(g.kernel)
    got = run([v.to_numpy() for v in f.inputs.values()])
    assert_f32(got, f.oracle(f.numpy_inputs()))


def test_the_planned_launch_runs_gridded(cuda, dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.launch import TileLevel, TileMachine
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.tile import compile_tile

    machine = TileMachine((TileLevel("shared", 128, 101376),))
    f = flash_tile(T=512, E=64, OD=64, SI=2)
    (g,) = plan_region(f.naive, machine=machine).groups
    assert g.template == "flash" and g.launch
    run = compile_tile(g.kernel, g.launch)
    assert run.grid > 1
    got = run([v.to_numpy() for v in f.inputs.values()])
    assert_f32(got, f.oracle(f.numpy_inputs()))


def test_mask_derived_bounds_prune_bit_exactly(cuda, dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.launch import TileLevel, TileMachine
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.tile import compile_tile

    machine = TileMachine((TileLevel("shared", 128, 101376),))
    f = flash_tile(T=128, E=32, OD=32, SI=2)
    (g,) = plan_region(f.naive, machine=machine).groups
    assert g.prune == (("so", (0, 0, 1), (1, 1, 1)),)
    vals = [v.to_numpy() for v in f.inputs.values()]
    np.testing.assert_array_equal(compile_tile(g.kernel, g.launch)(vals), compile_tile(g.kernel, g.launch, g.prune)(vals))


def test_the_rowstat_layernorm_runs(cuda, dsl):
    from pdum.tl.dialect import run_region
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.gpt2 import gpt2

    from pdum_dsl_b200.tile import compile_tile

    pm = plan_model(gpt2().region)
    carve = next(c for c in pm.carves if c.group.template == "row-statistics")
    vals = _tensors(carve.kernel, np.random.default_rng(17))
    want = run_region(carve.kernel, list(vals))
    got = compile_tile(carve.group.kernel)([v.to_numpy() for v in vals])
    assert_f32(got, want.to_numpy(order=want.names))


def test_the_flash_artifacts_store_from_one_sweep(cuda, dsl):
    from pdum.tl.autodiff import grad
    from pdum.tl.dialect import run_region
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.tile import compile_tile

    f = flash_tile(T=8, E=4, OD=4, SI=2)
    out = f.naive.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(f.naive.params)}
    names[id(out)] = "out"
    plan = plan_model(grad(f.naive, "out", seed="dO", names=names).region)
    fl = next(c for c in plan.carves if c.group.template == "flash")
    run = compile_tile(fl.group.kernel)
    vals = _tensors(fl.kernel, np.random.default_rng(31))
    want = run_region(fl.kernel, list(vals))
    got = run([v.to_numpy() for v in vals])
    assert isinstance(got, tuple) and len(got) == 3
    for gv, w in zip(got, want):
        assert_f32(gv, w.to_numpy(order=w.names))


def test_config1_region_through_the_widened_plan(cuda, dsl):
    from pdum_dsl_b200.plan import plan_region
    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.tile import compile_tile

    spec, ins, (want,) = load("cfg1_flash_f32")
    region = attention_region(**spec["region"])
    (g,) = plan_region(region).groups
    assert g.template == "flash"
    assert_f32(compile_tile(g.kernel)(ins), want, what="config 1")


@pytest.mark.parametrize("case", ["causal_bf16_ragged", "gqa_bf16", "noncausal_bf16_kv_ragged"])
def test_bf16_regions_through_the_widened_plan(cuda, dsl, case):
    from pdum_dsl_b200.plan import plan_region
    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.tile import compile_tile

    spec, ins, outs = load(case)
    region = attention_region(**spec["region"])
    (g,) = plan_region(region).groups
    got = compile_tile(g.kernel, dtype="bf16")(ins)
    got = got if isinstance(got, tuple) else (got,)
    assert_bf16(got[0], outs[0], what=case)
    for gv, w in zip(got[1:], outs[1:]):
        np.testing.assert_allclose(gv, w, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("case", ["rowsoftmax_16x4096", "layernorm_37x1001"])
def test_row_regions_through_plan(cuda, dsl, case):
    from pdum_dsl_b200.plan import plan_region
    from pdum_dsl_b200.regions import layernorm_region, row_softmax_region
    from pdum_dsl_b200.tile import compile_tile

    spec, ins, (want,) = load(case)
    r = spec["region"]
    region = row_softmax_region(r["R"], r["C"]) if r["kind"] == "softmax" else layernorm_region(r["R"], r["C"], r["eps"])
    (g,) = plan_region(region).groups
    assert_f32(compile_tile(g.kernel)(ins), want, what=case)


def test_the_first_measurement_greens_the_group(cuda, dsl):
    """A measured fact lands in the reference's ledger keyed by (kernel content,
    machine) and is never re-measured warm (analysis.py:121-146), as the
    reference's own device test does for its Triton column."""
    import time
    from dataclasses import replace

    import torch
    from pdum.tl.analysis import defanalysis, no_reanalysis
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.tile import compile_tile

    f = flash_tile(T=256, E=64, OD=64, SI=2)
    (g,) = plan_region(f.naive).groups
    arrays = [v.to_numpy() for v in f.inputs.values()]

    @defanalysis("fusion.sm100a-ms", 1, ledger=True)
    def sm100_ms(kernel, *, machine, reps=10):
        run = compile_tile(kernel, dtype="bf16")
        run(arrays)
        laps = []
        for _ in range(reps):
            t0 = time.perf_counter()
            run(arrays)
            laps.append(time.perf_counter() - t0)
        return {"ms": sorted(laps)[len(laps) // 2] * 1e3, "reps": reps}

    machine = torch.cuda.get_device_name(0)
    fact = sm100_ms(g.kernel, machine=machine)
    assert fact.value["ms"] > 0
    with no_reanalysis():
        again = sm100_ms(g.kernel, machine=machine)
    assert again.key == fact.key
    assert replace(g, confidence="green").confidence == "green"


def test_the_tile_flagships_run(cuda, dsl):
    """The reference's hand-written tile flagships (zoo/tiles.py) through compile_tile,
    against their numpy oracles (conformance/test_triton_tile.py:27-35)."""
    from pdum.tl.zoo.tiles import flash_tile, gemm_tile

    from pdum_dsl_b200.tile import compile_tile

    for f in (flash_tile(), gemm_tile()):
        run = compile_tile(f.region)
        got = run([v.to_numpy() for v in f.inputs.values()])
        assert_f32(got, f.oracle(f.numpy_inputs()))


def test_ledger_measures_and_greens_planned_groups(cuda, dsl):
    """pdum_dsl_b200.ledger: the device time of each lowered group as a ledger fact
    (CUDA-event microseconds), the plan's groups green, and no re-measurement warm."""
    import torch
    from pdum.tl.analysis import no_reanalysis
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200 import ledger

    plan = plan_region(flash_tile(T=256, E=64, OD=64, SI=2).naive)
    machine = torch.cuda.get_device_name(0)
    green, facts = ledger.green_plan(plan, machine=machine, reps=5)
    assert [g.confidence for g in green.groups] == ["green"]
    assert 0 < facts[0].value["us"] < 1e5
    with no_reanalysis():
        again = ledger.sm100_us(plan.groups[0].kernel, machine=machine, dtype="bf16", reps=5)
    assert again.key == facts[0].key


@pytest.mark.parametrize("group", [None, 2])
def test_runner_host_path_pinned_buffers_and_out(cuda, dsl, group):
    """compile_tile's host call with pinned bf16 torch buffers and a caller-owned
    output (the pipelined host path) equals the device path bit for bit."""
    import torch

    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.tile import compile_tile

    H = 4
    region = attention_region(B=2, H=H if group is None else H // group, T=300, D=128, causal=True,
                              scale=0.088, group=group)
    run = compile_tile(region, dtype="bf16")
    g = torch.Generator().manual_seed(9)
    vals = [torch.randn(tuple(d.stop - d.start for d in p.type.dims), generator=g).to(torch.bfloat16).pin_memory()
            for p in region.params]
    yld = region.body[-1].args[0]
    out = torch.empty(tuple(d.stop - d.start for d in yld.type.dims), dtype=torch.bfloat16).pin_memory()
    assert run(vals, out=out) is out
    want = run.run_t(*[v.cuda() for v in vals]).cpu()
    assert torch.equal(out, want)
    got_np = run([v.float().numpy() for v in vals])  # the reference's numpy convention
    np.testing.assert_array_equal(got_np, want.float().numpy())
