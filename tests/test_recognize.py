"""Host logic: the recogniser, compile-time refusals and the widened plan_region (CPU)."""

import numpy as np
import pytest

from pdum_dsl_b200.recognize import AttentionSpec, RowSpec, Untranslatable, recognize


def test_flash_tile_naive_and_planned_kernel(dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    f = flash_tile()
    spec = recognize(f.naive)
    assert isinstance(spec, AttentionSpec) and spec.causal and spec.scale is None and spec.riders == ()
    (g,) = plan_region(f.naive).groups
    tspec = recognize(g.kernel)  # the generated online-softmax fold (fusion.py:542-615)
    assert tspec.source == "tile" and tspec.causal and (tspec.t, tspec.s, tspec.e, tspec.o) == ("t", "s", "e", "o")
    assert recognize(f.region).source == "tile"  # the hand-written tile flagship


@pytest.mark.parametrize("kw,expect", [
    (dict(B=2, H=3, T=8, D=4, causal=True, scale=0.5), dict(riders=("b", "h"), causal=True, scale=0.5)),
    (dict(B=1, H=4, T=8, D=4, causal=False, scale=0.125), dict(riders=("b", "h"), causal=False, scale=0.125)),
    (dict(B=1, H=2, T=8, D=4, causal=True, scale=0.125, group=2), dict(riders=("b", "g"), group="r")),
    (dict(H=2, T=8, S=12, D=4, causal=False), dict(riders=("h",), causal=False, scale=None)),
    (dict(T=8, D=4, causal=True, artifacts=True), dict(artifacts=True, stat_dims=("t",))),
])
def test_widened_attention_spellings(dsl, kw, expect):
    from pdum_dsl_b200.regions import attention_region

    spec = recognize(attention_region(**kw))
    for k, v in expect.items():
        assert getattr(spec, k) == v, (k, getattr(spec, k), v)


def test_rows_and_rowstat_carve(dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.gpt2 import gpt2

    from pdum_dsl_b200.regions import layernorm_region, row_softmax_region

    s = recognize(row_softmax_region(4, 7))
    assert isinstance(s, RowSpec) and s.kind == "softmax" and s.dim == "c"
    (g,) = plan_region(row_softmax_region(4, 7)).groups
    assert g.template == "row-normalization" and recognize(g.kernel).kind == "softmax"  # staged rows
    ln = recognize(layernorm_region(4, 7, eps=1e-5))
    assert ln.kind == "layernorm" and ln.gamma == 1 and ln.beta == 2 and ln.eps == 1e-5
    pm = plan_model(gpt2().region)  # the reference's device test subject (test_fusion_triton.py:223)
    carve = next(c for c in pm.carves if c.group.template == "row-statistics")
    rs = recognize(carve.group.kernel)
    assert rs.kind == "layernorm"


def test_refusals_name_the_reason(dsl):
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    b = Builder({**CORE_OPS, **TL_OPS})
    x = Tensor.from_numpy(np.zeros((4, 5)), ("m", "k"))
    px = b.param(0, tensor_type_of_layout(x.layout))
    y = b.emit("tl.pointwise", px, f="sin")  # no lowered template has sin
    region = Region(params=(px,), body=(b.emit("core.yield", y),))
    with pytest.raises(Untranslatable, match="no sm_100a template"):
        recognize(region)


def test_compile_tile_checks_launch_and_dtype(dsl):
    from pdum.tl.fusion import plan_region
    from pdum.tl.launch import TileLevel, TileMachine
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.tile import compile_tile

    machine = TileMachine((TileLevel("shared", 128, 101376),))
    f = flash_tile(T=128, E=32, OD=32, SI=2)
    (g,) = plan_region(f.naive, machine=machine).groups
    run = compile_tile(g.kernel, g.launch, g.prune)  # the reference's own launch / prune artifacts
    assert run.grid == 2 and "flash_f32_kernel" in run.source
    with pytest.raises(Untranslatable, match="not an output dim"):
        compile_tile(f.naive, (("s", 32),))
    assert "flash_fwd" in compile_tile(f.naive, dtype="bf16").source  # E=32: the 64-wide build, zero-filled
    with pytest.raises(Untranslatable, match="head dims"):
        compile_tile(flash_tile(T=128, E=20, OD=20, SI=2).naive, dtype="bf16")  # rows not 16-byte multiples
    assert compile_tile(attention_region(T=300, D=64, causal=True), dtype="bf16").grid == 2


def test_widened_plan_region(dsl):
    from pdum_dsl_b200.plan import plan_region
    from pdum_dsl_b200.regions import attention_region

    for kw, mask in ((dict(B=1, H=2, T=200, D=64, causal=True, scale=0.125), "causal"),
                     (dict(B=1, H=2, T=64, D=16, causal=False, scale=0.25), "none"),
                     (dict(B=1, H=2, T=64, D=16, causal=True, scale=0.25, group=2), "causal"),
                     (dict(H=2, T=96, D=16, causal=True, window=40, scale=0.25), "intervals"),
                     (dict(B=2, T=96, D=16, causal=False, block=32, scale=0.25), "intervals")):
        (g,) = plan_region(attention_region(**kw)).groups
        assert g.template == "flash" and g.confidence == "yellow"
        # certified on the widened region itself (its own online-softmax fold vs the region)
        assert g.certificate.verdict == "licensed-differential"
        assert "flash.online-softmax" in g.certificate.licenses
        assert g.certificate.families == ("gaussian", "wide-scores", "dominant-key")
        assert dict(g.params)["mask"] == mask
    from pdum_dsl_b200.regions import row_softmax_region

    (g,) = plan_region(row_softmax_region(4, 8)).groups  # untouched rows stay the reference's
    assert g.template == "row-normalization"


def test_widened_fold_is_the_region_on_every_family(dsl):
    """The generated fold of a widened region (riders, GQA group, scale, sliding mask)
    evaluates equal to the naive region under run_region (the certificate's differential,
    rerun here directly at a tight tolerance)."""
    import numpy as np
    from pdum.tl.dialect import run_region
    from pdum.tl.tensor import Tensor

    from pdum_dsl_b200.recognize import match_naive_attention
    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.widen import generate_widened_flash

    r = attention_region(B=2, H=2, T=48, D=8, causal=True, window=20, scale=0.3, group=2)
    tile = generate_widened_flash(r, match_naive_attention(r))
    rng = np.random.default_rng(0)
    vals = [Tensor.from_numpy(rng.standard_normal(tuple(d.stop for d in p.type.dims)),
                              tuple(d.name for d in p.type.dims)) for p in r.params]
    a, b = run_region(r, vals), run_region(tile, list(vals))
    np.testing.assert_allclose(b.to_numpy(order=a.names), a.to_numpy(order=a.names), rtol=1e-12, atol=1e-12)


def test_compile_grad_reads_the_autodiff_joint(dsl):
    from pdum.tl.autodiff import grad

    from pdum_dsl_b200.grad import compile_grad
    from pdum_dsl_b200.regions import attention_region

    r = attention_region(B=1, H=2, T=8, D=64, causal=True, scale=0.5)
    out = r.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(r.params)}
    names[id(out)] = "out"
    run = compile_grad(grad(r, "out", seed="dO", names=names))
    assert run.spec.causal and run.spec.scale == 0.5 and run.spec.riders == ("b", "h")


def _gemm_subject():
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.dsl.types import f64
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    b = Builder({**CORE_OPS, **TL_OPS})
    t = lambda shape, names: tensor_type_of_layout(Tensor.from_numpy(np.zeros(shape), names).layout)
    pa, pb, pc = b.param(0, t((6, 8), ("m", "k"))), b.param(1, t((8, 5), ("k", "n"))), b.param(2, t((5,), ("n",)))
    prod = b.emit("tl.pointwise", b.emit("tl.repeat_like", pa, pb), b.emit("tl.repeat_like", pb, pa), f="mul")
    z = b.emit("tl.reduce", prod, dims=("k",), f="sum")
    zb = b.emit("tl.pointwise", z, b.emit("tl.repeat_like", pc, z), f="add")
    y = b.emit("tl.pointwise", zb, b.emit("core.const", type=f64, value=0.0), f="maximum")
    return Region(params=(pa, pb, pc), body=(b.emit("core.yield", y),))


def test_contraction_epilogue_naive_and_tile(dsl):
    from pdum.tl.fusion import plan_region

    from pdum_dsl_b200.recognize import ContractSpec

    r = _gemm_subject()
    s = recognize(r)
    assert isinstance(s, ContractSpec) and (s.m, s.n, s.k) == (("m",), ("n",), ("k",))
    assert [e[0] for e in s.epilogue] == ["add", "maximum"] and s.epilogue[0][1].param == 2
    (g,) = plan_region(r).groups
    assert g.template == "contraction-epilogue"
    assert recognize(g.kernel) == s  # the generated fold reads the same


def test_map_chain_spec(dsl):
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.dsl.types import f64
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    from pdum_dsl_b200.recognize import MapSpec

    b = Builder({**CORE_OPS, **TL_OPS})
    px = b.param(0, tensor_type_of_layout(Tensor.from_numpy(np.zeros((3, 4)), ("r", "c")).layout))
    y = b.emit("tl.pointwise", b.emit("tl.pointwise", px, f="exp"), b.emit("core.const", type=f64, value=2.0), f="mul")
    s = recognize(Region(params=(px,), body=(b.emit("core.yield", y),)))
    assert isinstance(s, MapSpec) and [e[0] for e in s.steps] == ["exp", "mul"]


def _flash_joint(T=64, E=8, OD=8):
    from pdum.tl.autodiff import grad
    from pdum.tl.zoo.tiles import flash_tile

    region = flash_tile(T=T, E=E, OD=OD, SI=2).naive
    out = region.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(region.params)}
    names[id(out)] = "out"
    return grad(region, "out", seed="dO", names=names)


def test_backend_record_for_the_seam(dsl):
    """The reference's backend capability record (dsl/registry.py:56-70): the
    fingerprint carries the library version, render names the launch, compile returns
    the compile_tile runner, and the record registers in a registry."""
    from pdum.dsl.registry import Backend, Registry
    from pdum.tl.zoo.tiles import flash_tile

    from pdum_dsl_b200._lib import version
    from pdum_dsl_b200.backend import b200_backend

    be = b200_backend()
    assert isinstance(be, Backend) and be.fp == ("b200_sm100a", version())
    region = flash_tile(T=64, E=8, OD=8, SI=2).naive
    src = be.render(region)
    assert "pdb_flash_fwd" in src
    run = be.compile(src, "flash")
    assert isinstance(run.spec, AttentionSpec)
    reg = Registry()
    reg.register_backend(be)
    assert reg.backends["b200_sm100a"] is be
    with pytest.raises(Untranslatable):
        be.render(_rows_only_unsupported())


def _rows_only_unsupported():
    """A region with no template here: a full (rank-0) sum over a single param."""
    import numpy as np
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    b = Builder({**CORE_OPS, **TL_OPS})
    x = b.param(0, tensor_type_of_layout(Tensor.from_numpy(np.zeros((3, 4)), ("r", "c")).layout))
    y = b.emit("tl.reduce", x, dims=("r", "c"), f="sum")
    return Region(params=(x,), body=(b.emit("core.yield", y),))


def test_general_closed_masks_read_as_key_intervals(dsl):
    """Sliding-window, block-diagonal and the zoo's sliding_attention masks evaluate
    exactly to one run of visible keys per row (the reference plans them as flash,
    fusion.py:468-477,521); rows with no visible key and non-run rows are refused."""
    import numpy as np
    from pdum.tl.zoo.attention import sliding_attention

    from pdum_dsl_b200.recognize import KeyIntervals
    from pdum_dsl_b200.regions import attention_region

    t = np.arange(300)
    sp = recognize(sliding_attention(T=300, E=4, OD=4, W=70).region)
    assert not sp.causal and isinstance(sp.mask, KeyIntervals) and sp.mask.monotone
    assert np.array_equal(sp.mask.lo, np.maximum(t - 69, 0)) and np.array_equal(sp.mask.hi, t + 1)
    bl = recognize(attention_region(T=300, D=4, causal=False, block=64)).mask
    assert np.array_equal(bl.lo, (t // 64) * 64) and np.array_equal(bl.hi, np.minimum((t // 64 + 1) * 64, 300))
    blc = recognize(attention_region(T=300, D=4, causal=True, block=64)).mask
    assert np.array_equal(blc.hi, t + 1) and np.array_equal(blc.lo, (t // 64) * 64)
    # the causal mask still reads as causal (the dedicated kernels' fast path)
    assert recognize(attention_region(T=300, D=4, causal=True)).causal is True
    with pytest.raises(Untranslatable, match="sees no key"):
        recognize(attention_region(T=40, D=4, causal=True, window=0))
    with pytest.raises(Untranslatable, match="single runs"):
        recognize(_strided_mask_region())


def _strided_mask_region():
    """Attention whose mask keeps the even keys only (not one run per row)."""
    from pdum.dsl.types import f64

    from pdum_dsl_b200 import regions as R

    Builder, Region, OPS, _, _, _ = R._dsl()
    (qn, qs), (kn, ks), (vn, vs) = R.attention_shapes(None, None, 16, 16, 4, 4, None)
    b = Builder(OPS)
    pq, pk, pv = (b.param(i, R._ptype(sh, nm)) for i, (nm, sh) in enumerate(((qn, qs), (kn, ks), (vn, vs))))
    sc = R._contract(b, pq, pk, "e")
    two = b.emit("core.const", type=f64, value=2.0)
    si = b.emit("tl.iota", sc, name="s")
    half = b.emit("tl.pointwise", b.emit("tl.pointwise", si, two, f="div"), f="floor")
    even = b.emit("tl.pointwise", b.emit("tl.pointwise", half, two, f="mul"), si, f="eq")
    sc = b.emit("tl.pointwise", even, sc, b.emit("core.const", type=f64, value=-1e9), f="where")
    pr, _, _ = R._softmax(b, sc, "s")
    return Region(params=(pq, pk, pv), body=(b.emit("core.yield", R._contract(b, pr, pv, "s")),))
