"""Builders for the DSL regions this backend executes (user-program side).

These construct ordinary pdum.dsl ``Region`` objects with the reference's own
``Builder`` and ``tl.*`` vocabulary, spelled exactly as the reference's zoo
spells them, so that ``plan_region`` / ``run_region`` accept them unchanged:

* attention: ``contract(q, k, axis=e)`` -> optional ``* scale`` -> optional
  causal ``where(iota(s) <= iota(t), sc, -1e9)`` -> softmax over ``s`` ->
  ``contract(pr, v, axis=s)`` (``pdum/tl/zoo/attention.py:167-196``,
  ``pdum/tl/zoo/zoo_common.py:79-86``, ``pdum/tl/zoo/tiles.py:238-252``);
  batch/head rider dims are extra leading dims; GQA spells query heads as
  ``(g, r)`` and K/V over ``g`` only, broadcast over ``r`` by the contraction
  (``pdum/tl/zoo/llama.py:1-9,51-54``);
* row softmax (``zoo_common.py:79-82``) and two-pass layernorm with a gamma /
  beta epilogue (``zoo_common.py:56-60``).

The DSL is imported lazily: this module is only usable where pdum.dsl /
pdum.tl are importable (the reference's own Python environment).
"""

from __future__ import annotations

import numpy as np


def _dsl():
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.dsl.types import f64
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    return Builder, Region, {**CORE_OPS, **TL_OPS}, f64, tensor_type_of_layout, Tensor


def _ptype(shape, names):
    *_, ttl, Tensor = _dsl()
    return ttl(Tensor.from_numpy(np.zeros(shape), tuple(names)).layout)


def _contract(b, x, y, dim):
    prod = b.emit("tl.pointwise", b.emit("tl.repeat_like", x, y), b.emit("tl.repeat_like", y, x), f="mul")
    return b.emit("tl.reduce", prod, dims=(dim,), f="sum")


def _softmax(b, sm, dim):
    mx = b.emit("tl.reduce", sm, dims=(dim,), f="max")
    e = b.emit("tl.pointwise", b.emit("tl.pointwise", sm, b.emit("tl.repeat_like", mx, sm), f="sub"), f="exp")
    den = b.emit("tl.reduce", e, dims=(dim,), f="sum")
    return b.emit("tl.pointwise", e, b.emit("tl.repeat_like", den, e), f="div"), mx, den


def attention_shapes(B, H, T, S, D, DV, group=None):
    """(names, shape) per param q, k, v.  ``B``/``H`` None drop the rider;
    ``group`` (query heads per KV head) switches to the GQA spelling where
    ``H`` counts KV heads (``g``) and ``r = group``."""
    lead_q, lead_k = [], []
    if B is not None:
        lead_q.append(("b", B))
        lead_k.append(("b", B))
    if group is not None:
        lead_q += [("g", H), ("r", group)]
        lead_k += [("g", H)]
    elif H is not None:
        lead_q.append(("h", H))
        lead_k.append(("h", H))
    q = lead_q + [("t", T), ("e", D)]
    k = lead_k + [("s", S), ("e", D)]
    v = lead_k + [("s", S), ("o", DV)]
    return [(tuple(n for n, _ in x), tuple(e for _, e in x)) for x in (q, k, v)]


def attention_region(B=None, H=None, T=6, S=None, D=3, DV=None, *, causal=True, scale=None,
                     group=None, artifacts=False, all_true_mask=False, window=None, block=None):
    """The naive (materialised-softmax) attention region; returns the Region.

    ``artifacts=True`` yields the tuple ``(out, m, den)`` -- the flash
    template's artifact variant (``pdum/tl/fusion.py:480-497``).
    ``all_true_mask=True`` (non-causal only) spells "no mask" as a closed
    always-true mask ``where(iota(s) <= iota(s), sc, -1e9)``, the form the
    reference's strict flash matcher requires (``fusion.py:468-477``).
    ``window=W`` (with causal) is the zoo's sliding mask ``(s <= t) * (t - s < W)``
    (``zoo/attention.py:84-103``); ``block=Bk`` is the block-diagonal (chunked)
    mask ``floor(t / Bk) == floor(s / Bk)``, causal within the block when
    ``causal`` -- both closed iota forests."""
    Builder, Region, OPS, f64, _, _ = _dsl()
    S = T if S is None else S
    DV = D if DV is None else DV
    (qn, qs), (kn, ks), (vn, vs) = attention_shapes(B, H, T, S, D, DV, group)
    b = Builder(OPS)
    pq = b.param(0, _ptype(qs, qn))
    pk = b.param(1, _ptype(ks, kn))
    pv = b.param(2, _ptype(vs, vn))
    sc = _contract(b, pq, pk, "e")
    if scale is not None:
        sc = b.emit("tl.pointwise", sc, b.emit("core.const", type=f64, value=float(scale)), f="mul")
    mask = None
    if causal or all_true_mask:
        other = "t" if causal else "s"
        mask = b.emit("tl.pointwise", b.emit("tl.iota", sc, name="s"), b.emit("tl.iota", sc, name=other), f="le")
    if window is not None:
        lag = b.emit("tl.pointwise", b.emit("tl.iota", sc, name="t"), b.emit("tl.iota", sc, name="s"), f="sub")
        inwin = b.emit("tl.pointwise", lag, b.emit("core.const", type=f64, value=float(window)), f="lt")
        mask = inwin if mask is None else b.emit("tl.pointwise", mask, inwin, f="mul")
    if block is not None:
        bk = b.emit("core.const", type=f64, value=float(block))
        bt = b.emit("tl.pointwise", b.emit("tl.pointwise", b.emit("tl.iota", sc, name="t"), bk, f="div"), f="floor")
        bs = b.emit("tl.pointwise", b.emit("tl.pointwise", b.emit("tl.iota", sc, name="s"), bk, f="div"), f="floor")
        same = b.emit("tl.pointwise", bt, bs, f="eq")
        mask = same if mask is None else b.emit("tl.pointwise", mask, same, f="mul")
    if mask is not None:
        sc = b.emit("tl.pointwise", mask, sc, b.emit("core.const", type=f64, value=-1e9), f="where")
    pr, mx, den = _softmax(b, sc, "s")
    out = _contract(b, pr, pv, "s")
    if artifacts:
        out = b.emit("core.tuple", out, mx, den)
    return Region(params=(pq, pk, pv), body=(b.emit("core.yield", out),))


def placed_attention_region(B, H, T, D, *, world, bind="h", level="gpu", causal=True, scale=None,
                            group=None, gather=True, S=None, DV=None):
    """Attention with one rider dim split over a machine level, in the reference's
    global-view placement spelling (``pdum/tl/zoo/megatron.py:1-14,45-50``): the
    rider ``bind`` ("b", "h", or "g" for GQA KV groups) of extent X becomes
    ``(w, <bind>l)`` with ``w`` (extent ``world``) bound to ``level`` and
    ``<bind>l = X / world`` per device.  With ``gather`` the output merges
    ``(w, <bind>l)`` back into ``<bind>`` -- the merge of a bound part that
    ``placement.traffic`` prices as an all-gather (``tl/placement.py:170-181``).
    The denotation is the unplaced region's (placement is metadata)."""
    Builder, Region, OPS, f64, ttl, Tensor = _dsl()
    S = T if S is None else S
    DV = D if DV is None else DV
    (qn, qs), (kn, ks), (vn, vs) = attention_shapes(B, H, T, S, D, DV, group)
    if bind not in qn or bind not in kn or bind in ("t", "s", "e", "o", "r"):
        raise ValueError(f"bind must name a rider dim shared by q and k/v (b, h or g), got {bind!r}")
    loc = f"{bind}l"

    def placed(names, shape):
        i = names.index(bind)
        if shape[i] % world:
            raise ValueError(f"{bind}={shape[i]} is not a multiple of world={world}")
        n2 = names[:i] + ("w", loc) + names[i + 1:]
        s2 = shape[:i] + (world, shape[i] // world) + shape[i + 1:]
        t = Tensor.from_numpy(np.zeros(s2), n2).bind(w=level)
        return ttl(t.layout)

    b = Builder(OPS)
    pq = b.param(0, placed(qn, qs))
    pk = b.param(1, placed(kn, ks))
    pv = b.param(2, placed(vn, vs))
    sc = _contract(b, pq, pk, "e")
    if scale is not None:
        sc = b.emit("tl.pointwise", sc, b.emit("core.const", type=f64, value=float(scale)), f="mul")
    if causal:
        mask = b.emit("tl.pointwise", b.emit("tl.iota", sc, name="s"), b.emit("tl.iota", sc, name="t"), f="le")
        sc = b.emit("tl.pointwise", mask, sc, b.emit("core.const", type=f64, value=-1e9), f="where")
    pr, _, _ = _softmax(b, sc, "s")
    out = _contract(b, pr, pv, "s")
    if gather:
        out = b.emit("tl.merge", out, parts=("w", loc), name=bind)
    return Region(params=(pq, pk, pv), body=(b.emit("core.yield", out),))


def row_softmax_region(R, C):
    """softmax over the column dim ``c`` of X(r, c) (``zoo_common.py:79-82``)."""
    Builder, Region, OPS, *_ = _dsl()
    b = Builder(OPS)
    px = b.param(0, _ptype((R, C), ("r", "c")))
    pr, _, _ = _softmax(b, px, "c")
    return Region(params=(px,), body=(b.emit("core.yield", pr),))


def layernorm_region(R, C, eps=1e-5):
    """Two-pass layernorm over ``c`` with gamma/beta (``zoo_common.py:56-60``):
    ``(x - mu) / sqrt(mean((x - mu)^2) + eps) * g + b``."""
    Builder, Region, OPS, f64, *_ = _dsl()
    b = Builder(OPS)
    px = b.param(0, _ptype((R, C), ("r", "c")))
    pg = b.param(1, _ptype((C,), ("c",)))
    pb = b.param(2, _ptype((C,), ("c",)))
    mu = b.emit("tl.reduce", px, dims=("c",), f="mean")
    xc = b.emit("tl.pointwise", px, b.emit("tl.repeat_like", mu, px), f="sub")
    var = b.emit("tl.reduce", b.emit("tl.pointwise", xc, xc, f="mul"), dims=("c",), f="mean")
    sd = b.emit("tl.pointwise", b.emit("tl.pointwise", var, b.emit("core.const", type=f64, value=float(eps)),
                                        f="add"), f="sqrt")
    y = b.emit("tl.pointwise", xc, b.emit("tl.repeat_like", sd, xc), f="div")
    y = b.emit("tl.pointwise", y, b.emit("tl.repeat_like", pg, y), f="mul")
    y = b.emit("tl.pointwise", y, b.emit("tl.repeat_like", pb, y), f="add")
    return Region(params=(px, pg, pb), body=(b.emit("core.yield", y),))
