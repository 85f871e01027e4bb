"""The B200 per-program machine table drives the reference's launch ladder (propose /
feasible / footprint, pdum/tl/launch.py:75-124) for the flash template."""

import pytest


@pytest.mark.parametrize("T,E", [(512, 64), (4096, 128)])
def test_b200_machine_ladders_feasible_launches(dsl, T, E):
    from pdum.tl.fusion import plan_region
    from pdum.tl.launch import TileLevel, TileMachine, feasible, footprint, propose
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.plan import B200_SMEM_PER_CTA, b200_machine
    from pdum_dsl_b200.tile import compile_tile

    m = b200_machine()
    assert m.tightest() == B200_SMEM_PER_CTA
    f = flash_tile(T=T, E=E, OD=E, SI=2)
    (g,) = plan_region(f.naive, machine=m).groups
    assert g.template == "flash" and g.launch
    ok, fp = feasible(g.kernel, g.launch, m)
    assert ok and fp == footprint(g.kernel, g.launch) <= B200_SMEM_PER_CTA
    ladder = propose(g.kernel, m)
    assert ladder and all(feasible(g.kernel, launch, m)[0] for launch in ladder)
    # a part with the reference test's 99 KB of shared memory admits no more launches
    small = TileMachine((TileLevel("shared", 128, 101376),))
    assert len(propose(g.kernel, small)) <= len(ladder)
    run = compile_tile(g.kernel, g.launch)  # the planned launch is accepted (validated, recorded)
    assert run.grid >= 1
