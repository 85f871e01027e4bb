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
* ``certificate`` is the reference's own flash certificate
  (``certify`` with the ``flash.online-softmax`` license over the
  adversarial families, ``fusion.py:696-715``) of the strict single-head
  twin at the shrunk extents (<= 128, the reference's ``_CERT_CAP``): the
  riders are independent instances of that program and the scale is a
  pointwise factor on the scores, so the twin's online-softmax law is the
  one the widened row relies on;
* ``params`` records what was widened (riders, group, scale, causal).

Requires the reference DSL (pdum.dsl / pdum.tl) to be importable.
"""

from __future__ import annotations

from .recognize import Untranslatable, match_naive_attention
from .regions import attention_region
from .tile import B200_FP

_CERT_CAP = 128


def _twin_certificate(region, spec):
    from pdum.tl import fusion

    def ext(i, n):
        d = next(d for d in region.params[i].type.dims if d.name == n)
        return d.stop - d.start

    T = min(ext(spec.q, spec.t), _CERT_CAP)
    S = T if spec.causal else min(ext(spec.k, spec.s), _CERT_CAP)
    E = min(ext(spec.q, spec.e), _CERT_CAP)
    O = min(ext(spec.v, spec.o), _CERT_CAP)
    twin = attention_region(T=T, S=S, D=E, DV=O, causal=spec.causal, all_true_mask=not spec.causal)
    (g,) = fusion.plan_region(twin).groups
    if g.template != "flash":
        raise Untranslatable(f"the strict twin did not plan as flash: {g.reason}")
    return g.certificate


def plan_region(region, machine=None, floor: int = 1024):
    """The reference's plan_region, with the widened flash rows (see the module docstring)."""
    from pdum.tl import fusion

    plan = fusion.plan_region(region, machine=machine, floor=floor)
    if len(plan.groups) != 1 or plan.groups[0].template != "uncompiled":
        return plan
    try:
        spec = match_naive_attention(region)
        cert = _twin_certificate(region, spec)
    except Untranslatable:
        return plan
    params = (("riders", spec.riders), ("group", spec.group), ("scale", spec.scale), ("causal", spec.causal),
              ("backend", B200_FP))
    arts = ("m", "den") if spec.artifacts else ()
    return fusion.Plan((fusion.Group("flash", region, cert, "yellow", params=params, artifacts=arts),))
