"""``plan_region`` with the flash template widened to the shapes the kernels run.

The reference registry recognises flash attention only in its strict v1
spelling -- single head, causal mask, no score scale
(``pdum/tl/fusion.py:480-539``); batch/head riders, a ``1/sqrt(D)`` scale,
the unmasked case and GQA plan as ``uncompiled`` (red).  This wrapper calls
the reference's ``plan_region`` unchanged and, only where it returns a
single red group for a region ``recognize`` reads as attention, returns the
same ``Plan`` / ``Group`` objects with a ``flash`` group instead:

* ``kernel`` is the region itself, so ``run_region(group.kernel, ...)``
  remains the oracle and ``compile_tile(group.kernel)`` lowers it;
* ``certificate`` is the reference's own certificate (``certify`` with the
  ``flash.online-softmax`` license over its adversarial families,
  ``fusion.py:618-656,696-715``) of the widened region itself: the
  online-softmax fold spelled for its riders / group / scale / mask
  (``widen.generate_widened_flash``) against the region, on a twin clamped
  to 2 per rider and 128 per other dim (the reference's cap);
* ``params`` records what was widened (riders, group, scale, mask).

Requires the reference DSL (pdum.dsl / pdum.tl) to be importable.
"""

from __future__ import annotations

from .recognize import Untranslatable, match_naive_attention
from .tile import B200_FP

_CERTS: dict = {}


def _certificate(region, spec):
    """certify_widened, memoised by the region's content key (the reference keeps
    certificates as analysis facts, fusion.py:696-715)."""
    from .widen import certify_widened

    key = getattr(region.body[-1], "key", None)
    if key is None or key not in _CERTS:
        cert = certify_widened(region, spec)
        if key is None:
            return cert
        _CERTS[key] = cert
    return _CERTS[key]


# Per-CTA on-chip capacities of an sm_100a program (B200): dynamic shared
# memory up to 227 KB (232448 bytes) per CTA, moved in 128-byte swizzle rows;
# tensor memory 512 columns x 128 lanes x 4 bytes = 256 KB, allocated in
# 32-column steps (16 KB).
B200_SMEM_PER_CTA = 232448
B200_TMEM_PER_SM = 512 * 128 * 4


def b200_machine():
    """One sm_100a CTA as the reference's per-program machine table (``TileMachine`` of
    ``TileLevel`` rows, ``pdum/tl/launch.py:37-52``), for ``plan_region(region,
    machine=b200_machine())``: the reference's ``propose`` / ``feasible``
    (``launch.py:75-124``) then ladder launches against the B200's shared memory
    (the tightest level) instead of a smaller part's."""
    from pdum.tl.launch import TileLevel, TileMachine

    return TileMachine((TileLevel("shared", 128, B200_SMEM_PER_CTA), TileLevel("tmem", 128 * 4 * 32, B200_TMEM_PER_SM)))


def plan_region(region, machine=None, floor: int = 1024):
    """The reference's plan_region, with the widened flash rows (see the module docstring)."""
    from pdum.tl import fusion

    plan = fusion.plan_region(region, machine=machine, floor=floor)
    if len(plan.groups) != 1 or plan.groups[0].template != "uncompiled":
        return plan
    try:
        spec = match_naive_attention(region)
    except Untranslatable:
        return plan
    cert = _certificate(region, spec)
    mask = "causal" if spec.causal else ("intervals" if spec.mask is not None else "none")
    params = (("riders", spec.riders), ("group", spec.group), ("scale", spec.scale), ("mask", mask),
              ("backend", B200_FP))
    arts = ("m", "den") if spec.artifacts else ()
    return fusion.Plan((fusion.Group("flash", region, cert, "yellow", params=params, artifacts=arts),))


_CHART_OPS = ("tl.with_charts", "tl.strip_charts", "tl.simplify")


def _bare(node):
    while node.op in _CHART_OPS:
        node = node.args[0]
    return node


def _lowered(carve):
    """The compile_tile runner of a carve: its plan group's tile kernel when a
    template row lowers it, else the carve's canonical kernel (the naive
    region the group was planned from -- same denotation), which the
    score-space program family lowers.  Raises Untranslatable if neither does."""
    from .tile import compile_tile

    tried = []
    for k in (carve.group.kernel, carve.kernel):
        if k is None:
            continue
        try:
            return compile_tile(k), k
        except Untranslatable as e:
            tried.append(str(e))
    raise Untranslatable(f"carve {carve.root_op} ({carve.group.template}): " + " | ".join(tried))


def device_assignment(plan) -> list[str]:
    """Per carve of a ``plan_model`` ModelPlan (``pdum/tl/partition.py:586``):
    ``"device"`` when a kernel of the sm_100a library executes it (every
    carve of the attention joint, the red max-adjoint scan included), else
    the reason it is refused."""
    out = []
    for c in plan.carves:
        if c.root is None:
            out.append("none")
            continue
        try:
            _lowered(c)
            out.append("device")
        except Untranslatable as e:
            out.append(f"refused: {e}")
    return out


def execute_model_plan(plan, region, values):
    """Execute a carved plan carve by carve, the way the reference executes one
    (``tests/test_partition.py:124-193``): a carve runs once every boundary value
    it reads is known, on the sm_100a library (f32 IEEE column; boundary values
    stay on the device between carves).  ``values`` are CUDA tensors per region
    param in type-dim order; returns the yielded values as CUDA tensors in the
    yield's dim order, and the per-carve assignment.  A carve no kernel lowers
    raises ``Untranslatable`` before anything runs -- there is no evaluator
    fallback."""
    runners = [(_lowered(c) if c.root is not None else None) for c in plan.carves]
    vals = {id(p): v for p, v in zip(region.params, values)}
    dims = {id(p): tuple(d.name for d in p.type.dims) for p in region.params}

    def known(b):
        while id(b) not in vals and b.op in _CHART_OPS:
            b = b.args[0]
        return b

    def arranged(b, param):
        """A boundary value in the dim order the carve's param expects."""
        v, have = vals[id(b)], dims[id(b)]
        want = tuple(d.name for d in param.type.dims)
        return v if have == want else v.permute(*[have.index(n) for n in want])

    pending = [(i, c) for i, c in enumerate(plan.carves) if c.root is not None]
    progressed = True
    while pending and progressed:
        progressed = False
        for i, c in list(pending):
            bounds = [known(b) for b in c.bounds]
            if not all(id(b) in vals for b in bounds):
                continue
            run, kernel = runners[i]
            ins = [arranged(b, p) for b, p in zip(bounds, kernel.params)]
            got = run.run_t(*ins)
            got = got if isinstance(got, tuple) else (got,)
            y = kernel.body[-1].args[0]
            ynodes = y.args if y.op == "core.tuple" else (y,)
            for node, val, yn in zip((c.root, *c.artifacts), got, ynodes):
                names = tuple(d.name for d in yn.type.dims)
                for key in (id(node), id(_bare(node))):  # chart roots alias their bare value
                    vals[key] = val.float()
                    dims[key] = names
            pending.remove((i, c))
            progressed = True
    if pending:
        raise RuntimeError("plan stalled: a carve reads a boundary value no carve produces")
    y = region.body[-1].args[0]
    targets = y.args if y.op == "core.tuple" else (y,)
    return tuple(vals[id(known(t))] for t in targets), ["device"] * sum(c.root is not None for c in plan.carves)
