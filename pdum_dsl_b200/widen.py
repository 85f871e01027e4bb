"""Certificates for the widened flash rows.

The reference certifies every flash group by a licensed differential between
the online-softmax fold its generator emits and the naive region it was
planned from, over adversarial input families (``certify.certify``,
``pdum/tl/certify.py:240-282``; license ``FLASH_ONLINE_SOFTMAX``,
``licenses.py:49-63``; families ``fusion._score_families``, ``fusion.py:
618-656``), at extents clamped to 128 when the region is larger
(``fusion.py:693-747``).  Its generator only spells the strict single-head,
unscaled shape.  This module spells the same fold for the shapes the B200
rows widen to -- batch / head riders, a GQA query group, a constant score
scale, any closed mask or none -- and certifies the widened region itself
against it with the reference's own ``certify``, license and families:

* the fold runs over ``so`` key tiles of ``si`` keys; elements are q repeated
  over ``so`` and k, v (and the mask, rebuilt as a closed form over a zero
  lattice with the score dims) split along ``s``;
* the step carries ``(m, den, o)`` over the query's non-feature dims and
  applies the flashsm recurrence (``zoo/attention.py:40-46``): scores
  ``scale * q.k``, ``where(mask, ., fill)``, running max, rescale, sum, PV;
* two folds share the step for the ``o`` and ``den`` finals (three with the
  artifact ``m``), and ``out = o / den``.

The twin is the widened region with riders clamped to 2 and every other dim
to 128 (the reference's cap), so the differential stays seconds long.
"""

from __future__ import annotations

from .recognize import AttentionSpec, Untranslatable, names_of

_CAP = 128
_RIDER_CAP = 2


def _ops():
    from pdum.dsl.ops import CORE_OPS
    from pdum.tl.dialect import TL_OPS

    return {**CORE_OPS, **TL_OPS}


def _pick_si(extent: int) -> int:
    """Largest divisor of the key extent that is <= 32 and leaves >= 2 tiles."""
    for si in range(min(32, extent // 2), 0, -1):
        if extent % si == 0:
            return si
    return extent


def _rebuild(b, memo, n, OPS):
    if id(n) in memo:
        return memo[id(n)]
    args = tuple(_rebuild(b, memo, x, OPS) for x in n.args)
    explicit = {} if OPS[n.op].type_rule is not None else {"type": n.type}
    out = b.emit(n.op, *args, loc=n.loc, **explicit, **dict(n.attrs))
    memo[id(n)] = out
    return out


def shrink(region, caps: dict):
    """The same program over clamped extents: every dim named in ``caps`` (else
    ``_CAP``) stops at its cap.  Param types are re-derived, extent-carrying
    attrs (``tl.const`` dims, ``tl.repeat`` extents) clamped, every other node
    re-typed by its rule.  None when a param dim starts above zero."""
    import numpy as np
    from pdum.dsl.ir import Builder, Region
    from pdum.tl.dialect import tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    OPS = _ops()
    if any(d.start != 0 for p in region.params for d in p.type.dims):
        return None

    def cap(name, stop):
        return min(int(stop), caps.get(name, _CAP))

    b = Builder(OPS)
    memo: dict[int, object] = {}
    for i, p in enumerate(region.params):
        dims = p.type.dims
        shape = tuple(cap(d.name, d.stop) for d in dims)
        t = tensor_type_of_layout(Tensor.from_numpy(np.zeros(shape), tuple(d.name for d in dims)).layout)
        memo[id(p)] = b.param(i, t)

    def rebuild(n):
        if id(n) in memo:
            return memo[id(n)]
        args = tuple(rebuild(x) for x in n.args)
        attrs = dict(n.attrs)
        if n.op == "tl.const" and "dims" in attrs:
            attrs["dims"] = tuple((nm, (e[0], cap(nm, e[1])) if isinstance(e, tuple) else cap(nm, e))
                                  for nm, e in tuple(attrs["dims"]))
        if n.op == "tl.repeat" and "extent" in attrs:
            e, nm = attrs["extent"], attrs.get("name")
            attrs["extent"] = (e[0], cap(nm, e[1])) if isinstance(e, tuple) else cap(nm, e)
        explicit = {} if OPS[n.op].type_rule is not None else {"type": n.type}
        out = b.emit(n.op, *args, loc=n.loc, **explicit, **attrs)
        memo[id(n)] = out
        return out

    yld = rebuild(region.body[-1].args[0])
    return Region(params=tuple(memo[id(p)] for p in region.params), body=(b.emit("core.yield", yld),))


def _attention_nodes(region, spec: AttentionSpec):
    """(mask node | None, fill, out node) of a naive attention region."""
    from .recognize import contract_core, f_of, softmax_core

    yld = region.body[-1].args[0]
    if yld.op == "core.tuple":
        yld = yld.args[0]
    x, y, _ = contract_core(yld)
    pr = x if y.op == "core.param" else y
    node = softmax_core(pr)["sm"]
    if f_of(node) == "where" and len(node.args) == 3:
        mask, _, fill = node.args
        return mask, float(dict(fill.attrs)["value"]), yld
    return None, -1e9, yld


def generate_widened_flash(region, spec: AttentionSpec):
    """The online-softmax fold (tile tier) of a widened naive attention region."""
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.types import f64
    from pdum.tl.dialect import _minus_dim, check_tier

    OPS = _ops()
    mask, fill, out_node = _attention_nodes(region, spec)
    qp, kp, vp = (region.params[i] for i in (spec.q, spec.k, spec.v))
    S = next(d.stop - d.start for d in kp.type.dims if d.name == spec.s)
    si = _pick_si(S)
    so = S // si
    qdims = [d for d in qp.type.dims if d.name != spec.e]  # the state dims (riders, [group], t)
    odim = next(d for d in vp.type.dims if d.name == spec.o)
    b = Builder(OPS)
    newp = {id(p): b.param(i, p.type) for i, p in enumerate(region.params)}
    nq, nk, nv = newp[id(qp)], newp[id(kp)], newp[id(vp)]
    els = [b.emit("tl.repeat", nq, name="so", extent=so), b.emit("tl.split", nk, name=spec.s, parts=(("so", so), ("si", si))),
           b.emit("tl.split", nv, name=spec.s, parts=(("so", so), ("si", si)))]
    if mask is not None:
        # the closed mask over a zero lattice with the score dims (its iota values, never data)
        sdims = tuple((d.name, d.stop) for d in qdims) + ((spec.s, S),)
        if any(d.start for d in qdims):
            raise Untranslatable("mask lattice needs query dims that start at 0")
        lattice = b.emit("tl.const", value=0.0, dims=sdims)
        memo = dict(newp)
        stack = [mask]
        while stack:
            n = stack.pop()
            if n.op == "tl.iota" and id(n) not in memo:
                memo[id(n)] = b.emit("tl.iota", lattice, name=dict(n.attrs)["name"])
            stack.extend(n.args)
        mk = _rebuild(b, memo, mask, OPS)
        if set(names_of(mk)) != {d[0] for d in sdims}:
            mk = b.emit("tl.repeat_like", mk, lattice)
        els.append(b.emit("tl.split", mk, name=spec.s, parts=(("so", so), ("si", si))))
    sdim_pairs = tuple((d.name, d.stop) for d in qdims)
    m0 = b.emit("tl.const", value=-1e30, dims=sdim_pairs)
    den0 = b.emit("tl.const", value=0.0, dims=sdim_pairs)
    o0 = b.emit("tl.const", value=0.0, dims=sdim_pairs + ((spec.o, odim.stop),))

    sb = Builder(OPS)
    p_m, p_den, p_o = sb.param(0, m0.type), sb.param(1, den0.type), sb.param(2, o0.type)
    p_els = [sb.param(3 + i, _minus_dim(e.type, "so")) for i, e in enumerate(els)]
    p_q, p_k, p_v = p_els[:3]
    ks = sb.emit("tl.stage", p_k, level="shared")
    vs = sb.emit("tl.stage", p_v, level="shared")
    prod = sb.emit("tl.pointwise", sb.emit("tl.repeat_like", p_q, ks), sb.emit("tl.repeat_like", ks, p_q), f="mul")
    sc = sb.emit("tl.reduce", prod, dims=(spec.e,), f="sum")
    if spec.scale is not None:
        sc = sb.emit("tl.pointwise", sc, sb.emit("core.const", type=f64, value=float(spec.scale)), f="mul")
    if mask is not None:
        pm = p_els[3]
        if names_of(pm) != names_of(sc):
            pm = sb.emit("tl.repeat_like", pm, sc)
        sc = sb.emit("tl.pointwise", pm, sc, sb.emit("core.const", type=f64, value=fill), f="where")
    m_new = sb.emit("tl.pointwise", p_m, sb.emit("tl.reduce", sc, dims=("si",), f="max"), f="maximum")
    alpha = sb.emit("tl.pointwise", sb.emit("tl.pointwise", p_m, m_new, f="sub"), f="exp")
    p_w = sb.emit("tl.pointwise", sb.emit("tl.pointwise", sc, sb.emit("tl.repeat_like", m_new, sc), f="sub"), f="exp")
    den_new = sb.emit("tl.pointwise", sb.emit("tl.pointwise", p_den, alpha, f="mul"),
                      sb.emit("tl.reduce", p_w, dims=("si",), f="sum"), f="add")
    pv = sb.emit("tl.pointwise", sb.emit("tl.repeat_like", p_w, vs), sb.emit("tl.repeat_like", vs, p_w), f="mul")
    o_new = sb.emit("tl.pointwise", sb.emit("tl.pointwise", p_o, sb.emit("tl.repeat_like", alpha, p_o), f="mul"),
                    sb.emit("tl.reduce", pv, dims=("si",), f="sum"), f="add")
    step = Region(params=(p_m, p_den, p_o, *p_els),
                  body=(sb.emit("core.yield", sb.emit("core.tuple", m_new, den_new, o_new)),))
    fold_args = (m0, den0, o0, *els)
    kw = dict(dim="so", state=("m", "den", "o"), element=("q", "k", "v", "mask")[:len(els)])
    f_o = b.emit("tl.fold", *fold_args, regions=(step,), out=("final", 2), **kw)
    f_den = b.emit("tl.fold", *fold_args, regions=(step,), out=("final", 1), **kw)
    out = b.emit("tl.pointwise", f_o, b.emit("tl.repeat_like", f_den, f_o), f="div")
    if spec.artifacts:
        f_m = b.emit("tl.fold", *fold_args, regions=(step,), out=("final", 0), **kw)
        out = b.emit("core.tuple", out, f_m, f_den)
    fused = Region(params=tuple(newp[id(p)] for p in region.params), body=(b.emit("core.yield", out),))
    return check_tier(fused, "tile")


def certify_widened(region, spec: AttentionSpec):
    """The reference's certificate (licensed differential, FLASH_ONLINE_SOFTMAX,
    its three adversarial families) of the widened region's own online-softmax
    fold against the region, on the clamped twin."""
    from pdum.tl.certify import certify
    from pdum.tl.fusion import _score_families
    from pdum.tl.licenses import FLASH_ONLINE_SOFTMAX

    from .recognize import match_naive_attention

    caps = {n: _RIDER_CAP for n in spec.riders}
    if spec.group:
        caps[spec.group] = _RIDER_CAP
    twin = shrink(region, caps)
    if twin is None:
        twin = region
    tspec = match_naive_attention(twin)
    tile = generate_widened_flash(twin, tspec)
    return certify(tile, twin, licenses=FLASH_ONLINE_SOFTMAX, families=_score_families(twin))
