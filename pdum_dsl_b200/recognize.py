"""Recognise the hot-path regions this backend executes (host logic, no DSL import).

Works on any object with the shape of pdum.dsl's IR (``Region.params``,
``Region.body``; ``Node.op / .args / .attrs / .regions / .type.dims`` with
dims carrying ``name / start / stop``), so the reference's own regions are
read as they are.  Three families are recognised:

* attention -- the naive (materialised-softmax) spelling the reference's
  ``_match_flash`` accepts (``pdum/tl/fusion.py:480-539``), widened with
  rider dims (batch / head), a constant score scale, the unmasked case and
  GQA (a query-only rider); and the tile region that ``_generate_flash``
  emits for it (``fusion.py:542-615``): a ``tl.fold`` over ``so`` carrying
  ``(m, den, o)`` whose finals are divided;
* row softmax -- ``_match_softmax`` (``fusion.py:371-400``), staged or not;
* two-pass layernorm -- ``_match_rowstat`` (``fusion.py:403-443``) with an
  optional gamma / beta epilogue (``zoo_common.py:56-60``).

Anything else raises ``Untranslatable`` naming the reason, the refusal
convention of ``conformance/region_evaluator.py:40-41``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


class Untranslatable(Exception):
    """The region is not one this backend lowers (the reason is the message)."""


def attrs(n) -> dict:
    return dict(n.attrs)


def f_of(n) -> str:
    return attrs(n).get("f", "") if n.op == "tl.pointwise" else ""


def dims_of(n) -> tuple:
    d = getattr(n.type, "dims", None)
    if d is None:
        raise Untranslatable(f"non-tensor value {n.op}")
    return tuple(d)


def names_of(n) -> tuple[str, ...]:
    return tuple(d.name for d in dims_of(n))


def red_dims(n) -> tuple[str, ...]:
    d = attrs(n)["dims"]
    return (d,) if isinstance(d, str) else tuple(d)


def unstage(n):
    while n.op == "tl.stage":
        n = n.args[0]
    return n


def is_const(n) -> bool:
    return n.op in ("core.const", "tl.const")


def const_value(n) -> float:
    return float(attrs(n)["value"])


def contract_core(n):
    """reduce(sum over one dim, mul(rl(x, y), rl(y, x))) -> (x, y, dim) or None."""
    if n.op != "tl.reduce":
        return None
    a = attrs(n)
    if a.get("f") != "sum" or a.get("zero") is not None:
        return None
    rd = red_dims(n)
    if len(rd) != 1:
        return None
    prod = n.args[0]
    if f_of(prod) != "mul" or len(prod.args) != 2:
        return None
    ra, rb = prod.args
    if ra.op != "tl.repeat_like" or rb.op != "tl.repeat_like":
        return None
    x, y = ra.args[0], rb.args[0]
    if ra.args[1] is not y or rb.args[1] is not x:
        return None
    return unstage(x), unstage(y), rd[0]


def softmax_core(pr):
    """div(exp(sm - rl(max_d sm)), rl(sum_d exp(...))) -> dict(sm, dim, max, den) or None."""
    if f_of(pr) != "div" or len(pr.args) != 2:
        return None
    e, rld = pr.args
    if f_of(e) != "exp" or rld.op != "tl.repeat_like":
        return None
    den = rld.args[0]
    if den.op != "tl.reduce" or attrs(den).get("f") != "sum" or den.args[0] is not e:
        return None
    sub = e.args[0]
    if f_of(sub) != "sub" or len(sub.args) != 2:
        return None
    sm, rlm = sub.args
    if rlm.op != "tl.repeat_like":
        return None
    mx = rlm.args[0]
    if mx.op != "tl.reduce" or attrs(mx).get("f") != "max" or mx.args[0] is not sm:
        return None
    if red_dims(den) != red_dims(mx) or len(red_dims(den)) != 1:
        return None
    return {"sm": sm, "dim": red_dims(den)[0], "max": mx, "den": den}


# --------------------------------------------------------------- mask forests
_CMP = {"le": np.less_equal, "lt": np.less, "ge": np.greater_equal, "gt": np.greater, "eq": np.equal,
        "ne": np.not_equal, "add": np.add, "sub": np.subtract, "mul": np.multiply, "maximum": np.maximum,
        "minimum": np.minimum, "and": np.logical_and, "or": np.logical_or, "div": np.true_divide}
_UNARY_MASK = {"floor": np.floor, "abs": np.abs, "neg": np.negative}


def _eval_mask(n, grid: dict):
    """Evaluate a closed mask forest (iota / const / pointwise) on coordinate grids."""
    if n.op == "tl.iota":
        name = attrs(n)["name"]
        if name not in grid:
            raise Untranslatable(f"mask reads coordinate {name!r}")
        return grid[name]
    if is_const(n):
        return const_value(n)
    if n.op == "tl.repeat_like":
        return _eval_mask(n.args[0], grid)
    if n.op == "tl.pointwise":
        f = f_of(n)
        vals = [_eval_mask(a, grid) for a in n.args]
        if f in _CMP and len(vals) == 2:
            return _CMP[f](vals[0], vals[1])
        if f == "not" and len(vals) == 1:
            return np.logical_not(vals[0])
        if f in _UNARY_MASK and len(vals) == 1:
            return _UNARY_MASK[f](vals[0])
        if f == "where" and len(vals) == 3:
            return np.where(vals[0], vals[1], vals[2])
        raise Untranslatable(f"mask op {f!r}")
    raise Untranslatable(f"mask node {n.op!r} reads data")


class KeyIntervals:
    """A closed mask read as one run of visible keys per query row: row t (relative
    to the query dim's start) sees keys lo[t] <= s < hi[t].  ``monotone`` when lo
    and hi are both nondecreasing (causal, sliding-window and block-local masks),
    which lets the kernels bound each block of rows' key tiles by its edge rows."""

    __slots__ = ("lo", "hi", "monotone")

    def __init__(self, lo, hi):
        self.lo = np.ascontiguousarray(lo, dtype=np.int32)
        self.hi = np.ascontiguousarray(hi, dtype=np.int32)
        self.monotone = bool(np.all(np.diff(self.lo) >= 0) and np.all(np.diff(self.hi) >= 0))

    def __repr__(self):
        return f"KeyIntervals(rows={len(self.lo)}, monotone={self.monotone})"


_ROW_CHUNK_ELEMS = 1 << 22


def classify_mask(mask, t: str, s: str, t_range: tuple[int, int], s_range: tuple[int, int]):
    """Evaluate a closed mask forest exactly over the whole (t, s) grid.

    Returns True when it is causal (s <= t in absolute coordinates), False when
    it is all-true, else the ``KeyIntervals`` of a mask whose every row's visible
    keys form one run.  Refuses (Untranslatable) a row with no visible key --
    the reference gives such a row uniform-softmax semantics and refuses to
    prune it (fusion.py:659-687) -- and rows whose visible keys are not one run."""
    if f_of(mask) == "le" and all(a.op == "tl.iota" for a in mask.args):
        if (attrs(mask.args[0])["name"], attrs(mask.args[1])["name"]) == (s, t) and s_range[0] == 0:
            if s_range[1] >= t_range[1]:  # every row sees keys 0..t
                return True
    if f_of(mask) == "ge" and all(a.op == "tl.iota" for a in mask.args):
        if (attrs(mask.args[0])["name"], attrs(mask.args[1])["name"]) == (t, s) and s_range[0] == 0:
            if s_range[1] >= t_range[1]:
                return True
    (t0, t1), (s0, s1) = t_range, s_range
    ss = np.arange(s0, s1, dtype=np.int64)
    S = len(ss)
    chunk = max(1, _ROW_CHUNK_ELEMS // max(S, 1))
    los, his = [], []
    for a in range(t0, t1, chunk):
        ts = np.arange(a, min(a + chunk, t1), dtype=np.int64)
        grid = {t: ts[:, None], s: ss[None, :]}
        m = np.broadcast_to(np.asarray(_eval_mask(mask, grid), dtype=bool), (len(ts), S))
        any_ = m.any(axis=1)
        if not any_.all():
            bad = int(ts[np.argmin(any_)])
            raise Untranslatable(f"mask row {t}={bad} sees no key (uniform-softmax semantics; not lowered)")
        lo = m.argmax(axis=1)
        hi = S - m[:, ::-1].argmax(axis=1)
        if not np.array_equal(m.sum(axis=1), hi - lo):
            raise Untranslatable("mask rows are not single runs of visible keys")
        los.append(lo + s0)
        his.append(hi + s0)
    lo = np.concatenate(los)
    hi = np.concatenate(his)
    if (lo == s0).all() and (hi == s1).all():
        return False
    tabs = np.arange(t0, t1)
    if s0 == 0 and (lo == 0).all() and np.array_equal(hi, np.minimum(tabs + 1, s1)) and s1 >= t1:
        return True
    return KeyIntervals(lo, hi)


# ------------------------------------------------------------------ attention
@dataclass(frozen=True)
class AttentionSpec:
    q: int  # param indices
    k: int
    v: int
    q_dims: tuple
    k_dims: tuple
    v_dims: tuple
    t: str
    s: str
    e: str
    o: str
    riders: tuple  # rider dims shared by q, k, v (k's order)
    group: str | None  # GQA query-only rider
    scale: float | None
    causal: bool
    artifacts: bool
    out_dims: tuple
    stat_dims: tuple  # dims of the m / den artifacts
    t_start: int
    source: str  # "naive" | "tile"
    mask: KeyIntervals | None = None  # a general closed mask (causal is then False)


def _param_index(region, n):
    for i, p in enumerate(region.params):
        if p is n:
            return i
    return None


def _strip_scale(sc):
    """mul(sc, c) / mul(c, sc) / div(sc, c) -> (sc, scale); else (sc, None)."""
    f = f_of(sc)
    if f == "mul" and len(sc.args) == 2:
        a, b = sc.args
        if is_const(b) and not is_const(a):
            return a, const_value(b)
        if is_const(a) and not is_const(b):
            return b, const_value(a)
    if f == "div" and len(sc.args) == 2 and is_const(sc.args[1]):
        return sc.args[0], 1.0 / const_value(sc.args[1])
    return sc, None


def _attention_dims(region, q, k, v, e, s, t_hint=None):
    qi, ki, vi = (_param_index(region, x) for x in (q, k, v))
    if None in (qi, ki, vi):
        raise Untranslatable("q, k and v must be region params")
    qd, kd, vd = names_of(q), names_of(k), names_of(v)
    if e not in qd or e not in kd or s not in kd or s not in vd:
        raise Untranslatable("score / value contraction dims do not line up")
    riders_k = tuple(n for n in kd if n not in (s, e))
    o_cand = [n for n in vd if n not in (s,) + riders_k]
    if len(o_cand) != 1 or set(vd) != set(riders_k) | {s, o_cand[0]}:
        raise Untranslatable(f"v dims {vd} are not (riders..., s, o)")
    q_rest = [n for n in qd if n != e and n not in riders_k]
    if len(q_rest) == 1:
        t, group = q_rest[0], None
    elif len(q_rest) == 2:
        if t_hint is None or t_hint not in q_rest:
            raise Untranslatable("cannot tell the query dim from the GQA rider")
        t = t_hint
        group = next(n for n in q_rest if n != t)
    else:
        raise Untranslatable(f"q dims {qd}: expected (riders..., [group], t, e)")
    if len(riders_k) > 2:
        raise Untranslatable(f"at most two shared rider dims (batch, head), got {riders_k}")
    if any(d.start != 0 for d in dims_of(k)):
        raise Untranslatable("k / v dims must start at 0 (the s coordinate is absolute)")
    tdim = next(d for d in dims_of(q) if d.name == t)
    return qi, ki, vi, qd, kd, vd, t, o_cand[0], riders_k, group, tdim.start


def match_naive_attention(region, yld=None) -> AttentionSpec:
    """``yld`` (default: the region's yield) is the node to read as attention."""
    yld = region.body[-1].args[0] if yld is None else yld
    artifacts = False
    m_out = den_out = None
    if yld.op == "core.tuple":
        if len(yld.args) != 3:
            raise Untranslatable("tuple yield is not (out, m, den)")
        yld, m_out, den_out = yld.args
        artifacts = True
    cc = contract_core(yld)
    if cc is None:
        raise Untranslatable("output is not a contraction")
    x, y, s = cc
    pr, v = (x, y) if y.op == "core.param" else (y, x)
    sm = softmax_core(pr)
    if sm is None or sm["dim"] != s:
        raise Untranslatable("contraction operand is not a softmax over the contracted dim")
    if artifacts and (m_out is not sm["max"] or den_out is not sm["den"]):
        raise Untranslatable("surfaced statistics are not the softmax's own (m, den)")
    node = sm["sm"]
    mask = None
    if f_of(node) == "where" and len(node.args) == 3:
        mask, node, fill = node.args
        if not is_const(fill):
            raise Untranslatable("mask fill is not a constant")
        if const_value(fill) > -1e4:
            raise Untranslatable("mask fill must be a large negative constant (masked scores carry no weight)")
    node, scale = _strip_scale(node)
    core = contract_core(node)
    if core is None:
        raise Untranslatable("scores are not a contraction")
    a, b, e = core
    q, k = (a, b) if s in names_of(b) else (b, a)
    qdims_only = [n for n in names_of(q) if n not in names_of(k)]
    out_dims = names_of(yld)
    t_hint = _pick_t(out_dims, qdims_only, names_of(v))
    qi, ki, vi, qd, kd, vd, t, o, riders, group, t_start = _attention_dims(region, q, k, v, e, s, t_hint)
    causal, kmask = False, None
    if mask is not None:
        tdim = next(d for d in dims_of(q) if d.name == t)
        sdim = next(d for d in dims_of(k) if d.name == s)
        causal = classify_mask(mask, t, s, (tdim.start, tdim.stop), (sdim.start, sdim.stop))
        if isinstance(causal, KeyIntervals):
            causal, kmask = False, causal
    return AttentionSpec(qi, ki, vi, qd, kd, vd, t, s, e, o, riders, group, scale, causal, artifacts, out_dims,
                         names_of(m_out) if artifacts else (), t_start, "naive", kmask)


def _pick_t(out_dims, q_only, v_dims):
    """The query dim is q-only and in the output; with GQA there are two such
    dims -- the query dim is the one adjacent to the value dim (t, o)."""
    cands = [n for n in q_only if n in out_dims]
    if len(cands) == 1:
        return cands[0]
    o = [n for n in out_dims if n in v_dims and n not in q_only]
    if o:
        i = out_dims.index(o[-1])
        if i > 0 and out_dims[i - 1] in cands:
            return out_dims[i - 1]
    return cands[-1] if cands else None


def match_flash_tile(region) -> AttentionSpec:
    """The tile region _generate_flash emits (fusion.py:542-615)."""
    yld = region.body[-1].args[0]
    artifacts = False
    f_m = None
    if yld.op == "core.tuple":
        if len(yld.args) != 3:
            raise Untranslatable("tuple yield is not (out, m, den)")
        yld, f_m, f_den_a = yld.args
        artifacts = True
    if f_of(yld) != "div" or len(yld.args) != 2:
        raise Untranslatable("tile output is not o / den")
    f_o, rl = yld.args
    if f_o.op != "tl.fold" or rl.op != "tl.repeat_like" or rl.args[0].op != "tl.fold":
        raise Untranslatable("tile output is not built from fold finals")
    f_den = rl.args[0]
    a_o, a_den = attrs(f_o), attrs(f_den)
    if tuple(a_o.get("state", ())) != ("m", "den", "o") or tuple(a_o.get("out", ())) != ("final", 2):
        raise Untranslatable("fold does not carry the online-softmax state (m, den, o)")
    if tuple(a_den.get("out", ())) != ("final", 1) or f_den.regions[0] is not f_o.regions[0]:
        raise Untranslatable("den final does not share the o fold's step")
    if artifacts and (f_m.op != "tl.fold" or tuple(attrs(f_m).get("out", ())) != ("final", 0)
                      or f_den_a is not f_den):
        raise Untranslatable("artifacts are not the fold's (m, den) finals")
    m0, den0, o0, qr, kt, vt, mt = f_o.args
    if not (is_const(m0) and const_value(m0) <= -1e29 and is_const(den0) and const_value(den0) == 0.0
            and is_const(o0) and const_value(o0) == 0.0):
        raise Untranslatable("fold initial state is not flashsm's identity (-1e30, 0, 0)")
    if qr.op != "tl.repeat" or kt.op != "tl.split" or vt.op != "tl.split" or mt.op != "tl.split":
        raise Untranslatable("fold element sources are not (repeat(q), split(k), split(v), split(mask))")
    q, k, v, mask = qr.args[0], kt.args[0], vt.args[0], mt.args[0]
    s = attrs(kt)["name"]
    step = f_o.regions[0]
    fill, e = _check_flash_step(step)
    if fill > -1e4:
        raise Untranslatable("mask fill must be a large negative constant")
    out_dims = names_of(yld)
    qi, ki, vi, qd, kd, vd, t, o, riders, group, t_start = _attention_dims(region, q, k, v, e, s)
    tdim = next(d for d in dims_of(q) if d.name == t)
    sdim = next(d for d in dims_of(k) if d.name == s)
    causal = classify_mask(mask, t, s, (tdim.start, tdim.stop), (sdim.start, sdim.stop))
    kmask = None
    if isinstance(causal, KeyIntervals):
        causal, kmask = False, causal
    return AttentionSpec(qi, ki, vi, qd, kd, vd, t, s, e, o, riders, group, None, causal, artifacts, out_dims,
                         names_of(f_m) if artifacts else (), t_start, "tile", kmask)


def _check_flash_step(step):
    """Verify the fold step is the flashsm step; return (fill, feature dim)."""
    body = step.body[-1].args[0]
    if body.op != "core.tuple" or len(body.args) != 3:
        raise Untranslatable("fold step does not yield (m, den, o)")
    m_new, den_new, o_new = body.args
    if f_of(m_new) != "maximum" or m_new.args[0] is not step.params[0]:
        raise Untranslatable("step m' is not max(m, max_si sm)")
    red = m_new.args[1]
    if red.op != "tl.reduce" or attrs(red).get("f") != "max":
        raise Untranslatable("step m' is not max(m, max_si sm)")
    sm = red.args[0]
    if f_of(sm) != "where" or sm.args[0] is not step.params[6] or not is_const(sm.args[2]):
        raise Untranslatable("step scores are not where(mask, sc, fill)")
    core = contract_core(sm.args[1])
    if core is None or core[0] is not step.params[3] or core[1] is not step.params[4]:
        raise Untranslatable("step scores are not contract(q, k_tile)")
    if f_of(den_new) != "add" or f_of(o_new) != "add":
        raise Untranslatable("step den' / o' are not rescale-and-add")
    return const_value(sm.args[2]), core[2]


def match_attention(region) -> AttentionSpec:
    """Naive or tile spelling; raises Untranslatable with the naive reason otherwise."""
    try:
        return match_naive_attention(region)
    except Untranslatable as naive_err:
        try:
            return match_flash_tile(region)
        except Untranslatable:
            raise naive_err from None


# -------------------------------------------------------------- row reductions
@dataclass(frozen=True)
class RowSpec:
    kind: str  # "softmax" | "layernorm"
    x: int
    gamma: int | None
    beta: int | None
    eps: float
    dim: str
    x_dims: tuple
    out_dims: tuple


def _rowstat_core(pr):
    """div(xc, rl(sqrt(mean(xc*xc) + eps))), xc = x - rl(mean(x)) -> (x, dim, eps) or None."""
    if f_of(pr) != "div" or len(pr.args) != 2:
        return None
    xc, rld = pr.args
    if rld.op != "tl.repeat_like":
        return None
    sd = rld.args[0]
    if f_of(sd) != "sqrt":
        return None
    add = sd.args[0]
    if f_of(add) != "add" or len(add.args) != 2:
        return None
    var, eps = add.args
    if is_const(var) and not is_const(eps):
        var, eps = eps, var
    if not is_const(eps) or var.op != "tl.reduce" or attrs(var).get("f") != "mean":
        return None
    sq = var.args[0]
    if f_of(sq) != "mul" or sq.args[0] is not sq.args[1] or sq.args[0] is not xc:
        return None
    if f_of(xc) != "sub" or len(xc.args) != 2:
        return None
    x, rlm = xc.args
    if rlm.op != "tl.repeat_like":
        return None
    mu = rlm.args[0]
    if mu.op != "tl.reduce" or attrs(mu).get("f") != "mean" or mu.args[0] is not x:
        return None
    if red_dims(var) != red_dims(mu) or len(red_dims(var)) != 1:
        return None
    return unstage(x), red_dims(var)[0], const_value(eps)


def _epilogue(node, op):
    """op(y, rl(p, y)) or op(rl(p, y), y) -> (y, param node) else None."""
    if f_of(node) != op or len(node.args) != 2:
        return None
    a, b = node.args
    if b.op == "tl.repeat_like" and unstage(b.args[0]).op == "core.param":
        return a, unstage(b.args[0])
    if a.op == "tl.repeat_like" and unstage(a.args[0]).op == "core.param":
        return b, unstage(a.args[0])
    return None


def match_rows(region) -> RowSpec:
    yld = region.body[-1].args[0]
    out_dims = names_of(yld)
    sm = softmax_core(yld)
    if sm is not None:
        x = unstage(sm["sm"])
        xi = _param_index(region, x)
        if xi is None:
            raise Untranslatable("row softmax operand is not a region param")
        return RowSpec("softmax", xi, None, None, 0.0, sm["dim"], names_of(x), out_dims)
    node, beta, gamma = yld, None, None
    ep = _epilogue(node, "add")
    if ep is not None:
        node, beta = ep
    ep = _epilogue(node, "mul")
    if ep is not None:
        node, gamma = ep
    core = _rowstat_core(node)
    if core is None:
        raise Untranslatable("not a row softmax or two-pass layernorm")
    x, dim, eps = core
    xi = _param_index(region, x)
    if xi is None:
        raise Untranslatable("layernorm operand is not a region param")
    gi = _param_index(region, gamma) if gamma is not None else None
    bi = _param_index(region, beta) if beta is not None else None
    for p in (gamma, beta):
        if p is not None and names_of(p) != (dim,):
            raise Untranslatable("gamma / beta must be vectors over the normalised dim")
    return RowSpec("layernorm", xi, gi, bi, eps, dim, names_of(x), out_dims)


def recognize(region):
    """-> AttentionSpec | RowSpec | ContractSpec, or raise Untranslatable."""
    errs = []
    for name, fn in (("attention", match_attention), ("rows", match_rows), ("contraction", lambda r: match_any_contraction(r)), ("map-chain", lambda r: match_map_chain(r))):
        try:
            return fn(region)
        except Untranslatable as e:
            errs.append(f"{name}: {e}")
    raise Untranslatable("no sm_100a template: " + "; ".join(errs))


# ------------------------------------------------------- contraction-epilogue
_UNARY = ("exp", "log", "sqrt", "tanh", "neg")
_BINARY = ("add", "sub", "mul", "div", "maximum", "minimum")


@dataclass(frozen=True)
class Leaf:
    """An epilogue operand: a constant, or a region param read at the output's coordinates."""

    const: float | None = None
    param: int | None = None
    dims: tuple = ()


@dataclass(frozen=True)
class ContractSpec:
    a: int  # param indices of the two operand params
    b: int
    a_pro: tuple  # unary prologue steps applied to the operand params (innermost first)
    b_pro: tuple
    a_dims: tuple
    b_dims: tuple
    k: tuple  # contracted dims
    batch: tuple  # kept dims shared by both operands
    m: tuple  # kept dims of a only
    n: tuple  # kept dims of b only
    mean: bool
    epilogue: tuple  # (op, Leaf | None, swap), applied from the accumulator outwards
    out_dims: tuple


def _contains(n, target, memo=None) -> bool:
    memo = {} if memo is None else memo
    if n is target:
        return True
    if id(n) in memo:
        return memo[id(n)]
    args = n.args[:1] if n.op == "tl.repeat_like" else n.args  # the "like" operand is shape only
    r = any(_contains(a, target, memo) for a in args)
    memo[id(n)] = r
    return r


def _leaf(region, n) -> Leaf | None:
    while n.op in ("tl.repeat_like", "tl.stage"):
        n = n.args[0]
    if is_const(n):
        return Leaf(const=const_value(n))
    i = _param_index(region, n)
    if i is not None:
        return Leaf(param=i, dims=names_of(n))
    return None


def _operand(region, x):
    """param, or a unary pointwise chain over a param -> (index, prologue, dims)."""
    pro = []
    while f_of(x) in _UNARY and len(x.args) == 1:
        pro.append(f_of(x))
        x = unstage(x.args[0])
    i = _param_index(region, x)
    if i is None:
        raise Untranslatable(f"contraction operand {x.op} is not a param or a unary chain over one")
    return i, tuple(reversed(pro)), names_of(x)


def match_contraction(region) -> ContractSpec:
    yld = region.body[-1].args[0]
    if yld.op == "core.tuple":
        raise Untranslatable("tuple yield")
    reduces = [n for n in _walk(region) if n.op == "tl.reduce"]
    if len(reduces) != 1:
        raise Untranslatable("a contraction-epilogue region has exactly one reduce")
    red = reduces[0]
    a_ = attrs(red)
    if a_.get("f") not in ("sum", "mean") or a_.get("zero") is not None:
        raise Untranslatable("the reduce is not a sum / mean")
    kdims = red_dims(red)
    prod = red.args[0]
    if f_of(prod) != "mul" or len(prod.args) != 2 or any(x.op != "tl.repeat_like" for x in prod.args):
        raise Untranslatable("the reduce is not over a broadcast product (the GEMM shape)")
    ra, rb = prod.args
    xa, xb = unstage(ra.args[0]), unstage(rb.args[0])
    if ra.args[1] is not rb.args[0] or rb.args[1] is not ra.args[0]:
        raise Untranslatable("the product is not the broadcast pair of two operands")
    ia, pa, da = _operand(region, xa)
    ib, pb, db = _operand(region, xb)
    if any(k not in da or k not in db for k in kdims):
        raise Untranslatable("both operands must carry the contracted dims")
    batch = tuple(n for n in da if n in db and n not in kdims)
    m = tuple(n for n in da if n not in db)
    n_ = tuple(n for n in db if n not in da)
    if da == db:
        raise Untranslatable("same-space operands (the rowsum shape) are not lowered")
    for x, dd in ((xa, da), (xb, db)):
        for d in dims_of(x):
            if d.start != 0:
                raise Untranslatable("operand dims must start at 0")
    # epilogue: a linear chain from the yield down to the reduce
    steps = []
    node = yld
    while node is not red:
        f = f_of(node)
        if f in _UNARY and len(node.args) == 1:
            steps.append((f, None, False))
            node = node.args[0]
            continue
        if f in _BINARY and len(node.args) == 2:
            l, r = node.args
            lc, rc = _contains(l, red), _contains(r, red)
            if lc == rc:
                raise Untranslatable("epilogue is not a chain over the accumulator")
            other = r if lc else l
            leaf = _leaf(region, other)
            if leaf is None:
                raise Untranslatable("epilogue operand is not a constant or a param")
            if leaf.param is not None and not set(leaf.dims) <= set(names_of(red)):
                raise Untranslatable("epilogue param has dims outside the output")
            steps.append((f, leaf, not lc))
            node = l if lc else r
            continue
        raise Untranslatable(f"epilogue step {node.op}/{f} is not lowered")
    if len(steps) > 8:
        raise Untranslatable("epilogue longer than 8 steps")
    return ContractSpec(ia, ib, pa, pb, da, db, kdims, batch, m, n_, a_.get("f") == "mean", tuple(reversed(steps)),
                        names_of(yld))


def _walk(region):
    seen, stack = set(), list(region.body)
    while stack:
        n = stack.pop()
        if id(n) in seen:
            continue
        seen.add(id(n))
        yield n
        stack.extend(n.args)
        for r in n.regions:
            stack.extend(r.body)


def match_contraction_tile(region) -> ContractSpec:
    """The tile region _generate_contraction emits (fusion.py:268-324): a fold
    over ``ko`` whose step adds reduce(sum over ki [+ rest], mul(rl(a), rl(b)))
    to the accumulator, operands split at k, the epilogue rebuilt over the
    fold's final (a mean's 1/N finalize is one more epilogue step)."""
    yld = region.body[-1].args[0]
    folds = [n for n in _walk(region) if n.op == "tl.fold"]
    if len(folds) != 1:
        raise Untranslatable("not a single-fold contraction tile")
    fold = folds[0]
    fa = attrs(fold)
    if tuple(fa.get("state", ())) != ("acc",) or tuple(fa.get("element", ())) != ("a", "b"):
        raise Untranslatable("fold is not the (acc | a, b) contraction fold")
    acc0, at, bt = fold.args
    if not is_const(acc0) or const_value(acc0) != 0.0 or at.op != "tl.split" or bt.op != "tl.split":
        raise Untranslatable("fold sources are not split operands")
    k = attrs(at)["name"]
    step = fold.regions[0]
    nxt = step.body[-1].args[0]
    if f_of(nxt) != "add" or nxt.args[0] is not step.params[0] or nxt.args[1].op != "tl.reduce":
        raise Untranslatable("fold step is not acc + reduce")
    part = nxt.args[1]
    rest = tuple(d for d in red_dims(part) if d != "ki")
    prod = part.args[0]
    if f_of(prod) != "mul" or any(x.op != "tl.repeat_like" for x in prod.args):
        raise Untranslatable("fold step is not the broadcast product")
    ia, pa, da = _operand(region, unstage(at.args[0]))
    ib, pb, db = _operand(region, unstage(bt.args[0]))
    kdims = (k,) + rest
    batch = tuple(n for n in da if n in db and n not in kdims)
    m = tuple(n for n in da if n not in db)
    n_ = tuple(n for n in db if n not in da)
    steps = []
    node = yld
    while node is not fold:
        f = f_of(node)
        if f in _UNARY and len(node.args) == 1:
            steps.append((f, None, False))
            node = node.args[0]
            continue
        if f in _BINARY and len(node.args) == 2:
            l, r = node.args
            lc, rc = _contains(l, fold), _contains(r, fold)
            if lc == rc:
                raise Untranslatable("epilogue is not a chain over the accumulator")
            leaf = _leaf(region, r if lc else l)
            if leaf is None:
                raise Untranslatable("epilogue operand is not a constant or a param")
            steps.append((f, leaf, not lc))
            node = l if lc else r
            continue
        raise Untranslatable(f"epilogue step {node.op}/{f} is not lowered")
    if len(steps) > 8:
        raise Untranslatable("epilogue longer than 8 steps")
    return ContractSpec(ia, ib, pa, pb, da, db, kdims, batch, m, n_, False, tuple(reversed(steps)), names_of(yld))


def match_any_contraction(region) -> ContractSpec:
    try:
        return match_contraction(region)
    except Untranslatable as e:
        try:
            return match_contraction_tile(region)
        except Untranslatable:
            raise e from None


# ---------------------------------------------------------------- map-chain
@dataclass(frozen=True)
class MapSpec:
    x: int  # the param at the bottom of the chain
    x_dims: tuple
    steps: tuple  # (op, Leaf | None, swap), innermost first
    out_dims: tuple


def match_map_chain(region) -> MapSpec:
    """A linear pointwise chain over one param (the map-chain row, fusion.py:
    847-858) whose other operands are constants or params broadcast to it."""
    yld = region.body[-1].args[0]
    if yld.op == "core.tuple":
        raise Untranslatable("tuple yield")
    steps = []
    node = yld
    while _param_index(region, unstage(node)) is None:
        node = unstage(node)
        f = f_of(node)
        if f in _UNARY and len(node.args) == 1:
            steps.append((f, None, False))
            node = node.args[0]
            continue
        if f in _BINARY and len(node.args) == 2:
            l, r = (unstage(a) for a in node.args)
            lp = l.op == "tl.repeat_like" or is_const(l)
            rp = r.op == "tl.repeat_like" or is_const(r)
            # the spine is the operand that is not a broadcast leaf / constant
            if not lp and (rp or _param_index(region, r) is not None):
                spine, other, swap = l, r, False
            elif not rp and (lp or _param_index(region, l) is not None):
                spine, other, swap = r, l, True
            else:
                raise Untranslatable("map chain is not linear")
            leaf = _leaf(region, other)
            if leaf is None:
                raise Untranslatable("map-chain operand is not a constant or a param")
            steps.append((f, leaf, swap))
            node = spine
            continue
        raise Untranslatable(f"map-chain step {node.op}/{f} is not lowered")
    x = unstage(node)
    if len(steps) > 8 or not steps:
        raise Untranslatable("map chain must have 1..8 steps")
    if set(names_of(x)) != set(names_of(yld)):
        raise Untranslatable("the chain's base param must span the output")
    return MapSpec(_param_index(region, x), names_of(x), tuple(reversed(steps)), names_of(yld))
