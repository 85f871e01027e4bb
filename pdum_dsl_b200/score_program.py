"""Score-space programs: the carves of the attention backward, lowered whole.

``plan_model`` (``pdum/tl/partition.py:586-607``) carves the joint region that
``autodiff.grad`` builds from the naive attention region.  Besides the flash
carve and plain GEMM carves it yields carves that re-derive the probabilities
inside the carve -- ``exp(where(mask, q.k, fill) - m) / den`` rebuilt from q, k
and the forward's statistics -- and then

* reduce a score-space expression over one score dim (the den-gradient and
  D-rowsum statistics: ``reduce_s(dP * div.d1(E, den))`` and friends),
* contract it with a matrix over one score dim (``dV^T[o, s] = sum_t P[t, s]
  dO[t, o]``), or
* yield the (t, s) tile itself (``dS``), and one red carve whose max-adjoint
  is spelled with a prefix count (``tl.scan``) to send the cotangent to the
  first maximal key only.

The reference serves these with its contraction-epilogue row
(``fusion.py:159-324``) or, for the red scan, with ``run_region``.  Here each
carve compiles into one or two launches of ``pdb_score_program_f32``: a
program of SSA steps evaluated per element of the score space (score
contractions, row / column vectors, iota coordinates, the pointwise markers
and the derivative markers ``f.dI`` of autodiff expanded into primitive
steps), followed by an output stage (store the tile, reduce each row, or
contract each row with a matrix).  The prefix-count idiom
``c * (scan_sum(where(c, 1, 0)) == 1)`` is exactly "c holds and no earlier
element along the scan dim holds c", i.e. ``iota == first index where c``;
it compiles to a pre-pass that takes that first index as a row minimum and
an equality in the main pass.

Recognition is structural and refuses (``Untranslatable``) anything outside
this form; there is no evaluator fallback.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .recognize import Untranslatable, attrs, const_value, dims_of, f_of, is_const, names_of, red_dims

_WRAPS = ("tl.with_charts", "tl.strip_charts", "tl.simplify", "tl.with_labels", "tl.stage")
_BIG = 1.0e30  # "no such index" for the first-index pre-pass

_BIN = {"add", "sub", "mul", "div", "maximum", "minimum", "le", "lt", "ge", "gt", "eq", "ne", "and", "or"}
_UN = {"exp", "log", "neg", "sqrt", "tanh", "abs", "not", "floor"}


def _unwrap(n):
    while n.op in _WRAPS:
        n = n.args[0]
    return n


@dataclass
class Pass:
    """One launch of pdb_score_program_f32 (host-side, before register allocation)."""

    rows: str  # the program's row dim
    cols: str  # the program's column dim (reduced / contracted when the mode reduces)
    batch: tuple = ()  # up to three rider dims (outer first): independent instances
    steps: list = field(default_factory=list)  # (kind, args tuple, value) SSA, index = value id
    scores: list = field(default_factory=list)  # (a_ref, b_ref, feature dim)
    rowvecs: list = field(default_factory=list)  # refs: ("param", i) | ("temp", k)
    colvecs: list = field(default_factory=list)
    tiles: list = field(default_factory=list)
    result: int = -1
    mode: str = "tile"  # tile | row_sum | row_max | row_min | row_contract
    out: tuple = ("final",)  # ("final",) | ("temp", k)
    w: tuple | None = None  # ("param", i) for row_contract
    x: str | None = None  # the contraction output's other dim
    # after allocation
    ops: list = field(default_factory=list)  # (opname, dst, a, b, c, value)
    n_regs: int = 0
    out_reg: int = 0


@dataclass
class ScoreProgramSpec:
    passes: list
    temps: list  # per temp: its dim names (the pass's riders, then the vector's dim)
    out_dims: tuple
    extents: dict  # dim name -> (start, stop)
    param_dims: list  # per region param: its dim names (type-dim order)
    source: str = ""


class _Compiler:
    def __init__(self, region):
        self.region = region
        self.pidx = {id(p): i for i, p in enumerate(region.params)}
        self.extents = {}
        for n in _walk(region):
            try:
                for d in dims_of(n):
                    self.extents.setdefault(d.name, (d.start, d.stop))
            except Untranslatable:
                pass
        self.passes: list[Pass] = []
        self.temps: list[str] = []

    # ------------------------------------------------------------ helpers
    def param(self, n):
        return self.pidx.get(id(_unwrap(n)))

    def factors(self, n):
        """A 3-D broadcast product -> its lower-dimensional factor nodes."""
        n = _unwrap(n)
        if n.op in ("tl.repeat", "tl.repeat_like"):
            x = _unwrap(n.args[0])
            return self.factors(x) if len(names_of(x)) == len(names_of(n)) else [x]
        f = f_of(n)
        if f == "mul" and len(n.args) == 2:
            return self.factors(n.args[0]) + self.factors(n.args[1])
        if f == "mul.d0" and len(n.args) == 2:
            return self.factors(n.args[1])
        if f == "mul.d1" and len(n.args) == 2:
            return self.factors(n.args[0])
        raise Untranslatable(f"3-D node {n.op}/{f} is not a broadcast product")

    # ------------------------------------------------------------ passes
    def new_pass(self, rows, cols, mode, batch=()):
        p = Pass(rows, cols, batch=tuple(batch), mode=mode)
        self.passes.append(p)
        return p

    def emit(self, p: Pass, memo: dict, n) -> int:
        n = _unwrap(n)
        key = id(n)
        if key in memo:
            return memo[key]
        v = self._emit(p, memo, n)
        memo[key] = v
        return v

    def step(self, p: Pass, kind, args=(), value=0.0) -> int:
        p.steps.append((kind, tuple(args), float(value)))
        return len(p.steps) - 1

    def const(self, p, value):
        return self.step(p, "const", (), value)

    def _slot(self, lst, ref):
        if ref not in lst:
            lst.append(ref)
        return lst.index(ref)

    def _emit(self, p: Pass, memo, n) -> int:
        R, Cc = p.rows, p.cols
        if is_const(n):
            return self.const(p, const_value(n))
        space = {R, Cc} | set(p.batch)
        i = self.pidx.get(id(n))
        if i is not None:
            dn = set(names_of(n))
            if not dn <= space:
                raise Untranslatable(f"param with dims {names_of(n)} in a {p.batch + (R, Cc)} program")
            if R in dn and Cc in dn:
                return self.step(p, "tile", (self._slot(p.tiles, ("param", i)),))
            if Cc in dn:
                return self.step(p, "col", (self._slot(p.colvecs, ("param", i)),))
            # over the rows, or over riders only (then constant along the rows: stride 0)
            return self.step(p, "row", (self._slot(p.rowvecs, ("param", i)),))
        dn = names_of(n)
        if not set(dn) <= space:
            if n.op == "tl.reduce":
                return self._score(p, n)
            raise Untranslatable(f"{n.op} with dims {dn} outside the score space ({R}, {Cc})")
        if n.op == "tl.iota":
            name = attrs(n)["name"]
            if name == R:
                return self.step(p, "iota_row")
            if name == Cc:
                return self.step(p, "iota_col")
            raise Untranslatable(f"iota over {name!r}")
        if n.op in ("tl.repeat", "tl.repeat_like"):
            return self.emit(p, memo, n.args[0])
        if n.op == "tl.reduce":
            return self._score(p, n)
        if n.op == "tl.pointwise":
            return self._pointwise(p, memo, n)
        raise Untranslatable(f"{n.op} is not a score-space step")

    def _score(self, p: Pass, n) -> int:
        a = attrs(n)
        rd = red_dims(n)
        if a.get("f") != "sum" or a.get("zero") is not None or len(rd) != 1:
            raise Untranslatable("an inner reduce must be a sum over one feature dim")
        f = rd[0]
        fac = [x for x in self.factors(n.args[0])]
        if len(fac) != 2:
            raise Untranslatable("score contraction is not a product of two operands")
        sides = {}
        for x in fac:
            i = self.param(x)
            dx = set(names_of(_unwrap(x)))
            if i is None or f not in dx:
                raise Untranslatable("score contraction operands must be params carrying the feature dim")
            own = dx & {p.rows, p.cols}
            if len(own) != 1 or not dx - own - {f} <= set(p.batch):
                raise Untranslatable("score contraction operands do not span the score space")
            other = own.pop()
            if other in sides:
                raise Untranslatable("score contraction operands do not span the score space")
            sides[other] = ("param", i)
        ref = (sides[p.rows], sides[p.cols], f)
        return self.step(p, "score", (self._slot(p.scores, ref),))

    def _pointwise(self, p: Pass, memo, n) -> int:
        f = f_of(n)
        # the first-index idiom: c * (scan_sum(where(c, 1, 0)) == 1)
        if f == "mul" and len(n.args) == 2:
            hit = self._first_index(p, memo, n)
            if hit is not None:
                return hit
        base, _, which = f.partition(".d")
        args = n.args
        if which:
            return self._slope(p, memo, base, int(which), args)
        ev = [self.emit(p, memo, a) for a in args]
        if base == "where" and len(ev) == 3:
            return self.step(p, "where", ev)
        if base in _BIN and len(ev) == 2:
            return self.step(p, base, ev)
        if base in _UN and len(ev) == 1:
            return self.step(p, base, ev)
        raise Untranslatable(f"pointwise {f!r} is not a score-space step")

    def _slope(self, p, memo, base, i, args) -> int:
        """The local slope marker f.dI (autodiff's derivative table, first-wins at kinks)."""
        e = lambda k: self.emit(p, memo, args[k])  # noqa: E731
        one = lambda: self.const(p, 1.0)  # noqa: E731
        if base in ("add",) or (base == "sub" and i == 0):
            return one()
        if (base == "sub" and i == 1) or base == "neg":
            return self.const(p, -1.0)
        if base == "mul":
            return e(1 - i)
        if base == "div":
            if i == 0:
                return self.step(p, "recip", (e(1),))
            b = e(1)
            return self.step(p, "neg", (self.step(p, "div", (e(0), self.step(p, "mul", (b, b)))),))
        if base == "exp":
            return self.step(p, "exp", (e(0),))
        if base == "log":
            return self.step(p, "recip", (e(0),))
        if base == "sqrt":
            return self.step(p, "recip", (self.step(p, "mul", (self.const(p, 2.0), self.step(p, "sqrt", (e(0),)))),))
        if base == "tanh":
            t = self.step(p, "tanh", (e(0),))
            return self.step(p, "sub", (one(), self.step(p, "mul", (t, t))))
        if base == "maximum":
            return self.step(p, "ge", (e(0), e(1))) if i == 0 else self.step(p, "gt", (e(1), e(0)))
        if base == "minimum":
            return self.step(p, "le", (e(0), e(1))) if i == 0 else self.step(p, "lt", (e(1), e(0)))
        if base == "abs":
            return self.step(p, "where", (self.step(p, "ge", (e(0), self.const(p, 0.0))), one(), self.const(p, -1.0)))
        if base == "where" and i in (1, 2):
            c = e(0)
            a, b = (one(), self.const(p, 0.0)) if i == 1 else (self.const(p, 0.0), one())
            return self.step(p, "where", (c, a, b))
        raise Untranslatable(f"slope marker {base}.d{i} is not lowered")

    def _first_index(self, p: Pass, memo, n):
        for c, z in (n.args, n.args[::-1]):
            c, z = _unwrap(c), _unwrap(z)
            if f_of(z) != "eq" or len(z.args) != 2:
                continue
            sc, one = (_unwrap(a) for a in z.args)
            if sc.op != "tl.scan" or not is_const(one) or const_value(one) != 1.0:
                continue
            sa = attrs(sc)
            if sa.get("f") != "sum":
                continue
            w = _unwrap(sc.args[0])
            if f_of(w) != "where" or len(w.args) != 3 or _unwrap(w.args[0]) is not c:
                continue
            if not (is_const(_unwrap(w.args[1])) and const_value(_unwrap(w.args[1])) == 1.0
                    and is_const(_unwrap(w.args[2])) and const_value(_unwrap(w.args[2])) == 0.0):
                continue
            dim = sa.get("dim")
            if dim not in (p.rows, p.cols):
                continue
            other = p.rows if dim == p.cols else p.cols
            # pre-pass over (other, dim): first index along dim where c holds, as a row minimum
            pre = self.new_pass(other, dim, "row_min", p.batch)
            pm: dict = {}
            cv = self.emit(pre, pm, c)
            idx = self.step(pre, "iota_col")
            pre.result = self.step(pre, "where", (cv, idx, self.const(pre, _BIG)))
            k = len(self.temps)
            self.temps.append(tuple(p.batch) + (other,))
            pre.out = ("temp", k)
            # keep the pre-pass ahead of the pass that reads it
            self.passes.remove(pre)
            self.passes.insert(self.passes.index(p), pre)
            if dim == p.cols:
                first = self.step(p, "row", (self._slot(p.rowvecs, ("temp", k)),))
                it = self.step(p, "iota_col")
            else:
                first = self.step(p, "col", (self._slot(p.colvecs, ("temp", k)),))
                it = self.step(p, "iota_row")
            return self.step(p, "eq", (it, first))
        return None


def _walk(region):
    seen, stack = set(), list(region.body)
    while stack:
        n = stack.pop()
        if id(n) in seen:
            continue
        seen.add(id(n))
        yield n
        stack.extend(n.args)


def _allocate(p: Pass, max_regs: int) -> None:
    """Linear-scan register allocation of the SSA steps (registers reused after last use)."""
    last = {}
    for i, (kind, args, _) in enumerate(p.steps):
        if kind not in ("score", "row", "col", "tile"):
            for a in args:
                last[a] = i
    last[p.result] = len(p.steps)
    free: list[int] = []
    reg = {}
    n_regs = 0
    p.ops = []
    for i, (kind, args, value) in enumerate(p.steps):
        if i not in last:  # dead value (e.g. an unused constant)
            continue
        src = tuple(reg[a] for a in args) if kind not in ("score", "row", "col", "tile") else args
        # free operands whose last use is this step before choosing dst
        if kind not in ("score", "row", "col", "tile"):
            for a in set(args):
                if last.get(a) == i:
                    free.append(reg[a])
        if kind == "score":
            # a score step writes its register cooperatively after a barrier; never alias an operand
            pass
        if free:
            free.sort()
            d = free.pop(0)
        else:
            d = n_regs
            n_regs += 1
        reg[i] = d
        a, b, c = (list(src) + [0, 0, 0])[:3]
        p.ops.append((kind, d, a, b, c, value))
    if n_regs > max_regs:
        raise Untranslatable(f"score program needs {n_regs} registers (at most {max_regs})")
    p.n_regs = max(1, n_regs)
    p.out_reg = reg[p.result]


def _largest(cands, extents, order):
    """The candidate dim with the largest extent (ties: the last in ``order``)."""
    cands = [d for d in order if d in cands]
    if not cands:
        raise Untranslatable("no row dim for the score-space program")
    return max(reversed(cands), key=lambda d: extents[d][1] - extents[d][0])


def match_score_program(region, max_ops: int = 64, max_regs: int = 12) -> ScoreProgramSpec:
    """The carve as score-space program passes.  The row dim is the kept score dim
    (the largest candidate), the column dim the reduced / contracted one (or the
    yield's last dim for a tile), and any remaining yield dims (at most three) are
    riders: independent instances, broadcast (stride 0) in operands that lack them."""
    yld = _unwrap(region.body[-1].args[0])
    if yld.op == "core.tuple":
        raise Untranslatable("tuple yield")
    comp = _Compiler(region)
    out_dims = names_of(yld)
    ext = comp.extents
    if yld.op == "tl.reduce":
        a = attrs(yld)
        rd = red_dims(yld)
        if a.get("zero") is not None or len(rd) != 1 or a.get("f") not in ("sum", "max", "min"):
            raise Untranslatable("output reduce is not a sum / max / min over one dim")
        s = rd[0]
        x = _unwrap(yld.args[0])
        xd = names_of(x)
        if len(xd) == len(out_dims) + 1 and set(out_dims) | {s} == set(xd) and _is_program(comp, x):
            t = _largest(set(xd) - {s}, ext, xd)
            p = comp.new_pass(t, s, "row_" + a["f"], tuple(d for d in out_dims if d != t))
            p.result = comp.emit(p, {}, x)
        elif a["f"] == "sum":
            fac = comp.factors(x)
            if len(fac) != 2 or any(s not in names_of(f) for f in fac):
                raise Untranslatable("contraction output is not (score-space expression) x (param matrix)")
            # the matrix operand is a param; the other factor is the score-space program
            order = sorted(fac, key=lambda f: comp.param(f) is not None)
            prog, mat = order
            if comp.param(mat) is None:
                raise Untranslatable("contraction output is not (score-space expression) x (param matrix)")
            pd, md = set(names_of(prog)), set(names_of(mat))
            xs = md - pd
            if len(xs) != 1:
                raise Untranslatable("the contraction's matrix operand must add exactly one output dim")
            xdim = xs.pop()
            t = _largest(pd - md - {s}, ext, names_of(prog))
            batch = tuple(d for d in out_dims if d not in (t, xdim))
            if set(out_dims) != {t, xdim} | set(batch) or not (pd | md) - {s, t, xdim} <= set(batch):
                raise Untranslatable("contraction output dims do not match its operands")
            p = comp.new_pass(t, s, "row_contract", batch)
            p.result = comp.emit(p, {}, prog)
            p.w, p.x = ("param", comp.param(mat)), xdim
        else:
            raise Untranslatable("output reduce is not over a score-space expression")
    elif len(out_dims) >= 2:
        p = comp.new_pass(out_dims[-2], out_dims[-1], "tile", out_dims[:-2])
        p.result = comp.emit(p, {}, yld)
    else:
        raise Untranslatable(f"yield of rank {len(out_dims)} is not a score-space program output")
    if any(len(ps.batch) > 3 for ps in comp.passes):
        raise Untranslatable("more than three rider dims")
    for ps in comp.passes:
        if len(ps.scores) > 2 or len(ps.rowvecs) > 6 or len(ps.colvecs) > 6 or len(ps.tiles) > 4:
            raise Untranslatable("score program reads more operands than the kernel takes")
        _allocate(ps, max_regs)
        if len(ps.ops) > max_ops:
            raise Untranslatable(f"score program of {len(ps.ops)} steps (at most {max_ops})")
    src = "; ".join(f"pass {k}: {ps.batch + (ps.rows, ps.cols)} {ps.mode} {len(ps.ops)} steps {ps.n_regs} regs "
                    f"{len(ps.scores)} contractions" for k, ps in enumerate(comp.passes))
    pdims = [names_of(p) for p in region.params]
    return ScoreProgramSpec(comp.passes, comp.temps, out_dims, comp.extents, pdims, "pdb_score_program_f32 " + src)


def _is_program(comp, x) -> bool:
    """True when x is an elementwise score-space expression (not a broadcast product
    to be contracted: those have a dim the output lacks besides the reduced one)."""
    x = _unwrap(x)
    if x.op in ("tl.repeat", "tl.repeat_like") or f_of(x) in ("mul", "mul.d0", "mul.d1"):
        try:
            fac = comp.factors(x)
        except Untranslatable:
            return True
        return not (len(fac) == 2 and any(comp.param(f) is not None for f in fac)
                    and len(names_of(x)) > max(len(names_of(f)) for f in fac))
    return True


# ------------------------------------------------------------------ execution
def run_score_program(spec: ScoreProgramSpec, tensors):
    """Device tensors per region param (type-dim order) -> the yield, a float32 device tensor."""
    import ctypes as C

    import torch

    from . import _lib

    ext = {k: v[1] - v[0] for k, v in spec.extents.items()}
    dev = tensors[0].device if tensors else torch.device("cuda", torch.cuda.current_device())
    ts = [t if t.dtype == torch.float32 else t.float() for t in tensors]
    temps = [torch.empty(tuple(ext[d] for d in dims), dtype=torch.float32, device=dev) for dims in spec.temps]
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    out = None

    def view(ref):
        kind, i = ref
        if kind == "param":
            return ts[i], spec.param_dims[i]
        return temps[i], spec.temps[i]

    def stride(ref, dim):
        t, names = view(ref)
        return t.stride(names.index(dim)) if dim in names else 0

    for ps in spec.passes:
        bd = list(ps.batch)
        while len(bd) < 3:
            bd.insert(0, None)

        def bstr(ref):
            return tuple(stride(ref, b) if b is not None else 0 for b in bd)

        d = _lib.ScoreProgramDesc()
        d.batch, d.batch_mid, d.batch_inner = (ext[b] if b is not None else 1 for b in bd)
        d.rows, d.cols = ext[ps.rows], ext[ps.cols]
        d.row_start, d.col_start = spec.extents[ps.rows][0], spec.extents[ps.cols][0]
        for k, (aref, bref, f) in enumerate(ps.scores):
            d.score_a[k], d.score_b[k] = view(aref)[0].data_ptr(), view(bref)[0].data_ptr()
            d.score_a_stride[k] = _lib.I64x5(*bstr(aref), stride(aref, ps.rows), stride(aref, f))
            d.score_b_stride[k] = _lib.I64x5(*bstr(bref), stride(bref, ps.cols), stride(bref, f))
            d.score_feat[k] = ext[f]
        d.n_scores = len(ps.scores)
        for k, ref in enumerate(ps.rowvecs):
            d.rowvec[k] = view(ref)[0].data_ptr()
            d.rowvec_stride[k] = _lib.I64x4(*bstr(ref), stride(ref, ps.rows))
        for k, ref in enumerate(ps.colvecs):
            d.colvec[k] = view(ref)[0].data_ptr()
            d.colvec_stride[k] = _lib.I64x4(*bstr(ref), stride(ref, ps.cols))
        for k, ref in enumerate(ps.tiles):
            d.tile[k] = view(ref)[0].data_ptr()
            d.tile_stride[k] = _lib.I64x5(*bstr(ref), stride(ref, ps.rows), stride(ref, ps.cols))
        for k, (kind, dst, a, b, c, value) in enumerate(ps.ops):
            o = d.ops[k]
            o.op, o.dst, o.a, o.b, o.c, o.value = _lib.SP_OPS[kind], dst, a, b, c, value
        d.n_ops, d.n_regs, d.result = len(ps.ops), ps.n_regs, ps.out_reg
        d.out_mode = _lib.SP_OUT[ps.mode]
        if ps.out[0] == "temp":
            o_t = temps[ps.out[1]]
            tref = ("temp", ps.out[1])
            d.out_stride = _lib.I64x5(*bstr(tref), stride(tref, ps.rows), 0)
        else:
            on = spec.out_dims
            o_t = torch.empty(tuple(ext[n] for n in on), dtype=torch.float32, device=dev)
            second = ps.cols if ps.mode == "tile" else ps.x if ps.mode == "row_contract" else None

            def ostr(n):
                return o_t.stride(on.index(n)) if n is not None and n in on else 0

            d.out_stride = _lib.I64x5(ostr(bd[0]), ostr(bd[1]), ostr(bd[2]), ostr(ps.rows), ostr(second))
            out = o_t
        d.out = o_t.data_ptr()
        if ps.mode == "row_contract":
            d.w = view(ps.w)[0].data_ptr()
            d.w_stride = _lib.I64x5(*bstr(ps.w), stride(ps.w, ps.cols), stride(ps.w, ps.x))
            d.xdim = ext[ps.x]
        _lib.check(lib.pdb_score_program_f32(C.byref(d), stream), "pdb_score_program_f32")
    return out
