"""Measurements of this backend as facts in the reference's analysis ledger.

The reference makes a group's confidence "green" only through a measurement:
an analysis declared ``ledger=True`` whose evaluator is the machine, keyed by
the kernel's content key plus the analysis fingerprint plus its parameters
(``pdum/tl/analysis.py:1-24,121-175``), so a keyed measurement is taken once
and reloaded, never repeated (``save_ledger`` / ``load_ledger``), and a warm
loop asserts zero re-analysis (``no_reanalysis``).  The reference's own device
test records its Triton column this way
(``conformance/test_fusion_triton.py:87-117``).

Here:

* ``sm100_us(kernel, machine=..., dtype=..., reps=...)`` -- the device time of
  ``compile_tile(kernel, dtype=dtype)`` in microseconds (CUDA events around
  back-to-back launches on seeded N(0,1) inputs drawn from the kernel's param
  types, median of ``reps``), a ledger fact;
* ``sm100_profile(kernel, facts, machine=...)`` -- profiler numbers (ncu
  counters such as DRAM bytes or tensor-pipe activity, taken outside the
  process) recorded against the same kernel key;
* ``green_plan(plan, machine=...)`` -- the plan with every group this backend
  lowers measured and marked green; groups it does not lower keep their
  confidence.

Requires the reference DSL (pdum.dsl / pdum.tl) to be importable.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np

_ANALYSES = {}


def _inputs(kernel, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(tuple(d.stop - d.start for d in p.type.dims)) for p in kernel.params]


def _time_us(kernel, dtype, reps):
    """Median device microseconds of one launch of the compiled kernel."""
    import torch

    from .tile import compile_tile

    run = compile_tile(kernel, dtype=dtype)
    arrays = _inputs(kernel)
    run(arrays)  # compiles nothing (prebuilt library) but checks the device path once
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    spec = run.spec
    tensors = []
    for i, a in enumerate(arrays):
        t = torch.as_tensor(a, dtype=torch.float32).cuda()
        if hasattr(spec, "q") and i in (spec.q, spec.k, spec.v):
            t = t.to(dt)
        tensors.append(t)
    for _ in range(3):
        run.run_t(*tensors)
    torch.cuda.synchronize()
    laps = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run.run_t(*tensors)
        e1.record()
        torch.cuda.synchronize()
        laps.append(e0.elapsed_time(e1) * 1e3)
    return sorted(laps)[len(laps) // 2]


def _analysis(name):
    if name in _ANALYSES:
        return _ANALYSES[name]
    from pdum.tl.analysis import defanalysis

    if name == "us":

        @defanalysis("fusion.sm100a-us", 1, ledger=True)
        def sm100a_us(kernel, *, machine, dtype, reps):
            return {"us": _time_us(kernel, dtype, reps), "reps": reps, "dtype": dtype, "machine": machine}

        _ANALYSES[name] = sm100a_us
    else:

        @defanalysis("fusion.sm100a-profile", 1, ledger=True)
        def sm100a_profile(kernel, *, machine, facts):
            return dict(facts, machine=machine)

        _ANALYSES[name] = sm100a_profile
    return _ANALYSES[name]


def sm100_us(kernel, *, machine: str, dtype: str = "bf16", reps: int = 20):
    """The ledger fact of this kernel's device time (see the module docstring)."""
    return _analysis("us")(kernel, machine=machine, dtype=dtype, reps=reps)


def sm100_profile(kernel, facts: dict, *, machine: str):
    """Record profiler numbers (plain JSON data) against the kernel key."""
    return _analysis("profile")(kernel, machine=machine, facts=dict(facts))


def green_plan(plan, *, machine: str, dtype: str = "bf16", reps: int = 20):
    """(plan with measured groups green, {group index: fact}).  A group is measured
    when this backend lowers its kernel; the rest keep their confidence."""
    from .recognize import Untranslatable
    from .tile import compile_tile

    groups, facts = [], {}
    for i, g in enumerate(plan.groups):
        if g.kernel is None or g.confidence == "red":
            groups.append(g)
            continue
        try:
            compile_tile(g.kernel, dtype=dtype)
        except Untranslatable:
            groups.append(g)
            continue
        facts[i] = sm100_us(g.kernel, machine=machine, dtype=dtype, reps=reps)
        groups.append(replace(g, confidence="green"))
    return replace(plan, groups=tuple(groups)), facts
