"""Contraction-epilogue template on silicon, mirroring the reference's device tests
(conformance/test_fusion_triton.py:54-66, :162-192, :250-269) with compile_tile."""

import numpy as np
import pytest

from tests.tolerances import assert_f32

pytestmark = pytest.mark.gpu


def _ops():
    from pdum.dsl.ops import CORE_OPS
    from pdum.tl.dialect import TL_OPS

    return {**CORE_OPS, **TL_OPS}


def _ptype(arr, names):
    from pdum.tl.dialect import tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    return tensor_type_of_layout(Tensor.from_numpy(arr, names).layout)


def _subject(M=6, K=8, N=5, seed=3):
    """relu(a @ b + bias) -- the epilogue-on-a-contraction case."""
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.types import f64

    rng = np.random.default_rng(seed)
    A, B, bias = rng.standard_normal((M, K)), rng.standard_normal((K, N)), rng.standard_normal(N)
    b = Builder(_ops())
    pa, pb, pc = b.param(0, _ptype(A, ("m", "k"))), b.param(1, _ptype(B, ("k", "n"))), b.param(2, _ptype(bias, ("n",)))
    prod = b.emit("tl.pointwise", b.emit("tl.repeat_like", pa, pb), b.emit("tl.repeat_like", pb, pa), f="mul")
    z = b.emit("tl.reduce", prod, dims=("k",), f="sum")
    zb = b.emit("tl.pointwise", z, b.emit("tl.repeat_like", pc, z), f="add")
    y = b.emit("tl.pointwise", zb, b.emit("core.const", type=f64, value=0.0), f="maximum")
    return Region(params=(pa, pb, pc), body=(b.emit("core.yield", y),)), [A, B, bias], np.maximum(A @ B + bias, 0.0)


@pytest.mark.parametrize("shape", [(6, 8, 5), (300, 257, 130)])
def test_fused_contraction_epilogue(cuda, dsl, shape):
    from pdum.tl.fusion import plan_region

    from pdum_dsl_b200.tile import compile_tile

    region, arrays, want = _subject(*shape)
    (g,) = plan_region(region).groups
    assert g.template == "contraction-epilogue"
    run = compile_tile(g.kernel)
    assert "contract_f32_kernel" in run.source
    assert_f32(run(arrays), want)
    assert_f32(compile_tile(region)(arrays), want)  # the naive spelling lowers the same


def test_computed_operand_prologue(cuda, dsl):
    from pdum.dsl.ir import Builder, Region
    from pdum.tl.fusion import plan_region

    from pdum_dsl_b200.tile import compile_tile

    rng = np.random.default_rng(9)
    X, dY = rng.standard_normal((32, 32)), rng.standard_normal((32, 16))
    b = Builder(_ops())
    px, pd = b.param(0, _ptype(X, ("t", "m"))), b.param(1, _ptype(dY, ("t", "n")))
    a = b.emit("tl.pointwise", px, f="exp")
    prod = b.emit("tl.pointwise", b.emit("tl.repeat_like", a, pd), b.emit("tl.repeat_like", pd, a), f="mul")
    y = b.emit("tl.reduce", prod, dims=("t",), f="sum")
    region = Region(params=(px, pd), body=(b.emit("core.yield", y),))
    (g,) = plan_region(region).groups
    run = compile_tile(g.kernel)
    assert_f32(run([X, dY]), np.exp(X).T @ dY)


def test_two_dim_contraction(cuda, dsl):
    from pdum.dsl.ir import Builder, Region
    from pdum.tl.fusion import plan_region

    from pdum_dsl_b200.tile import compile_tile

    rng = np.random.default_rng(23)
    X, W = rng.standard_normal((32, 4, 16)), rng.standard_normal((4, 16, 32))
    b = Builder(_ops())
    px, pw = b.param(0, _ptype(X, ("t", "nh", "hk"))), b.param(1, _ptype(W, ("nh", "hk", "d")))
    prod = b.emit("tl.pointwise", b.emit("tl.repeat_like", px, pw), b.emit("tl.repeat_like", pw, px), f="mul")
    y = b.emit("tl.reduce", prod, dims=("nh", "hk"), f="sum")
    region = Region(params=(px, pw), body=(b.emit("core.yield", y),))
    want = np.einsum("thk,hkd->td", X, W)
    assert_f32(compile_tile(region)([X, W]), want)
    (g,) = plan_region(region).groups
    assert_f32(compile_tile(g.kernel)([X, W]), want)


def test_bf16_tensor_core_contraction(cuda, dsl):
    """The tcgen05 path: bf16 operands (k contiguous), fp32 accumulate, bf16 out;
    the bar is bf16 output rounding: max err <= 2^-7 max|ref|."""
    from pdum_dsl_b200.tile import compile_tile
    from tests.golden import round_bf16

    region, _, _ = _subject(300, 264, 200)
    rng = np.random.default_rng(4)
    A, B, bias = (round_bf16(rng.standard_normal(s)) for s in ((300, 264), (264, 200), (200,)))
    run = compile_tile(region, dtype="bf16")
    assert "contract_bf16_kernel" in run.source
    want = np.maximum(A @ B + bias, 0)
    got = run([A, B, bias])
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()


def test_batched_bf16_contract_kernel(cuda):
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(2)
    a = torch.randn(3, 257, 192, generator=g).to(torch.bfloat16)
    b = torch.randn(3, 130, 192, generator=g).to(torch.bfloat16)
    bias = torch.randn(3, 1, 130, generator=g)
    c = kernels.contract(a.to(cuda), b.to(cuda), epilogue=[("mul", 0.5, False), ("add", bias.to(cuda), False),
                                                           ("tanh", None, False)])
    want = torch.tanh(0.5 * torch.einsum("bmk,bnk->bmn", a.double(), b.double()) + bias.double())
    assert (c.double().cpu() - want).abs().max() <= 2 ** -7


@pytest.mark.parametrize("shape", [(2, 600, 520, 200), (1, 1024, 768, 512), (1, 256, 256, 64)])
def test_pair_bf16_contract_kernel(cuda, monkeypatch, shape):
    """256 x 256 tiles on CTA pairs (cta_group::2): ragged M / N / K, a batch, the
    single-tile case; the single-CTA kernel on the same inputs must agree bit for bit
    (same k-order of the fp32 accumulation)."""
    import torch

    from pdum_dsl_b200 import kernels

    bsz, m, n, k = shape
    g = torch.Generator(device="cpu").manual_seed(11)
    a = torch.randn(bsz, m, k, generator=g).to(torch.bfloat16).to(cuda)
    b = torch.randn(bsz, n, k, generator=g).to(torch.bfloat16).to(cuda)
    bias = torch.randn(bsz, 1, n, generator=g).to(cuda)
    ep = [("add", bias, False), ("maximum", 0.0, False)]
    monkeypatch.setenv("PDB_CONTRACT_PAIR", "1")
    c_pair = kernels.contract(a, b, epilogue=ep)
    monkeypatch.setenv("PDB_CONTRACT_PAIR", "0")
    c_one = kernels.contract(a, b, epilogue=ep)
    kernels.check_device_errors()
    want = torch.relu(torch.einsum("bmk,bnk->bmn", a.double(), b.double()) + bias.double()).cpu()
    err = (c_pair.double().cpu() - want).abs().max().item()
    assert err <= 2 ** -7 * max(1.0, want.abs().max().item())
    assert torch.equal(c_pair, c_one)


def test_map_chain(cuda, dsl):
    """A pure pointwise chain (the map-chain row): y = tanh(x * 0.5 + b) - c, broadcast params."""
    from pdum.dsl.ir import Builder, Region
    from pdum.dsl.types import f64
    from pdum.tl.fusion import plan_region

    from pdum_dsl_b200.tile import compile_tile

    rng = np.random.default_rng(5)
    X, bvec, cmat = rng.standard_normal((37, 50)), rng.standard_normal(50), rng.standard_normal((37, 50))
    b = Builder(_ops())
    px, pb, pc = b.param(0, _ptype(X, ("r", "c"))), b.param(1, _ptype(bvec, ("c",))), b.param(2, _ptype(cmat, ("r", "c")))
    y = b.emit("tl.pointwise", px, b.emit("core.const", type=f64, value=0.5), f="mul")
    y = b.emit("tl.pointwise", y, b.emit("tl.repeat_like", pb, y), f="add")
    y = b.emit("tl.pointwise", y, f="tanh")
    y = b.emit("tl.pointwise", y, pc, f="sub")
    region = Region(params=(px, pb, pc), body=(b.emit("core.yield", y),))
    (g,) = plan_region(region).groups
    assert g.template == "map-chain"
    run = compile_tile(g.kernel)
    assert "pointwise" in run.source
    assert_f32(run([X, bvec, cmat]), np.tanh(X * 0.5 + bvec) - cmat)
