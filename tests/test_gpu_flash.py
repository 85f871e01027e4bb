"""Flash-attention forward kernels vs the reference's run_region fixtures and the oracle."""

import math

import numpy as np
import pytest

from oracle import attention as OA
from tests.golden import HERE, load
from tests.tolerances import assert_bf16, assert_f32

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32), device=dev).to(dtype)


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _flat_gqa(a, names):
    if "r" in names:
        return a.reshape(a.shape[0], a.shape[1] * a.shape[2], *a.shape[3:])
    return a


def test_flash_tile_flagship_f32(cuda):
    """The reference's own tile flagship (zoo/tiles.py:143), f32 column."""
    import torch

    from pdum_dsl_b200 import kernels

    z = np.load(HERE / "flash_tile_default.npz")
    o = kernels.flash_attention(_t(z["q"], cuda, torch.float32), _t(z["k"], cuda, torch.float32),
                                _t(z["v"], cuda, torch.float32), scale=1.0, causal=True)
    assert_f32(_np(o), z["naive"])


@pytest.mark.parametrize("case", ["cfg1_flash_f32", "causal_f32_small"])
def test_f32_flash_matches_reference(cuda, case):
    import torch

    from pdum_dsl_b200 import kernels

    spec, (q, k, v), (want, *_) = load(case)
    kw = spec["region"]
    o = kernels.flash_attention(_t(q, cuda, torch.float32), _t(k, cuda, torch.float32),
                                _t(v, cuda, torch.float32), scale=kw.get("scale") or 1.0, causal=kw["causal"])
    assert_f32(_np(o), want, what=case)


@pytest.mark.parametrize("case", ["causal_bf16_ragged", "causal_bf16_d128", "noncausal_bf16_kv_ragged", "gqa_bf16"])
def test_bf16_flash_matches_reference(cuda, case):
    import torch

    from pdum_dsl_b200 import kernels

    spec, (q, k, v), outs = load(case)
    kw = spec["region"]
    qn = spec["inputs"][0]["names"]
    q4 = _flat_gqa(q, qn)
    res = kernels.flash_attention(_t(q4, cuda, torch.bfloat16), _t(k, cuda, torch.bfloat16),
                                  _t(v, cuda, torch.bfloat16), scale=kw["scale"], causal=kw["causal"],
                                  return_artifacts=bool(kw.get("artifacts")))
    o = res[0] if isinstance(res, tuple) else res
    assert_bf16(_np(o).reshape(outs[0].shape), outs[0], what=case)
    if kw.get("artifacts"):
        m, den = _np(res[1]), _np(res[2])
        np.testing.assert_allclose(m.reshape(outs[1].shape), outs[1], rtol=1e-3, atol=1e-3)
        np.testing.assert_allclose(den.reshape(outs[2].shape), outs[2], rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("B,H,HKV,T,S,D,causal", [
    (1, 1, 1, 128, 128, 64, True), (1, 1, 1, 256, 256, 128, True), (2, 3, 3, 300, 300, 64, True),
    (1, 4, 1, 513, 513, 128, True), (1, 2, 2, 64, 1000, 128, False), (1, 1, 1, 1, 1, 64, False),
    (1, 2, 2, 1, 77, 64, True), (3, 2, 1, 257, 129, 64, False), (1, 2, 1, 300, 300, 256, True),
    (2, 2, 2, 129, 1000, 256, False), (1, 1, 1, 1, 1, 256, False), (1, 3, 3, 700, 700, 256, True)])
def test_bf16_shapes_vs_oracle(cuda, B, H, HKV, T, S, D, causal):
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(B * 1000 + T + S)
    q = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16)
    scale = 1 / math.sqrt(D)
    o, lse = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), scale=scale, causal=causal,
                                     return_lse=True)
    ro, _, _, rlse = OA.attention_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), scale=scale,
                                      causal=causal)
    assert_bf16(_np(o), ro)
    np.testing.assert_allclose(_np(lse), rlse, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_bf16_large_scores_rescale(cuda, D):
    """Wide scores (x8, the reference's adversarial family) and a dominant key row (x40):
    the running max jumps mid-row, so the O accumulator is rescaled."""
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(11)
    q = (8 * torch.randn(1, 2, 512, D, generator=g) * math.sqrt(64 / D)).to(torch.bfloat16)
    k = torch.randn(1, 2, 512, D, generator=g)
    k[:, :, 300] *= 40
    k = k.to(torch.bfloat16)
    v = torch.randn(1, 2, 512, D, generator=g).to(torch.bfloat16)
    for causal in (True, False):
        o = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), scale=0.125, causal=causal)
        ro, *_ = OA.attention_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), scale=0.125,
                                  causal=causal)
        assert_bf16(_np(o), ro)


def test_bf16_strided_inputs(cuda):
    """(B, T, H, D) storage read through strides, the layout torch's projections produce."""
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(5)
    qkv = torch.randn(2, 200, 3, 4, 128, generator=g).to(torch.bfloat16).to(cuda)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # (B, H, T, D) views
    o = kernels.flash_attention(q, k, v, causal=True)
    ro, *_ = OA.attention_fwd(*(x.double().cpu().numpy() for x in (q, k, v)), scale=1 / math.sqrt(128), causal=True)
    assert_bf16(_np(o), ro)


def _seeded(shape, seed, dev):
    """N(0,1) from numpy default_rng(seed) (one seed per tensor), rounded to bf16 on the device."""
    import torch

    a = np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
    return torch.from_numpy(a).to(dev).to(torch.bfloat16)


def test_bf16_config3_slices(cuda):
    """Config 3 (B8 H32 S4096 D128 causal): full-size launch from seeded draws (q, k, v:
    seeds 30, 31, 32); 16 heads spread over every batch vs the oracle, all heads finite."""
    import torch

    from pdum_dsl_b200 import kernels

    shape = (8, 32, 4096, 128)
    q, k, v = (_seeded(shape, 30 + i, cuda) for i in range(3))
    o = kernels.flash_attention(q, k, v, causal=True)
    kernels.check_device_errors()
    assert torch.isfinite(o).all()
    for b, h in [(b, (5 * b + 3 * j) % 32) for b in range(8) for j in range(2)]:
        ro, *_ = OA.attention_fwd(*(x[b, h].double().cpu().numpy() for x in (q, k, v)), scale=1 / math.sqrt(128),
                                  causal=True)
        assert_bf16(_np(o[b, h]), ro, what=f"head ({b},{h})")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_query_offset_rows_see_the_absolute_causal_mask(cuda, dtype):
    """A row slab t in [q_start, q_start + T) of a longer sequence (the reference's
    iota masks use absolute coordinates, dialect.py:1382-1383)."""
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(17)
    T, S, D, q_start = 200, 333, 64, 133
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    q = torch.randn(1, 2, T, D, generator=g).to(tdt)
    k = torch.randn(1, 2, S, D, generator=g).to(tdt)
    v = torch.randn(1, 2, S, D, generator=g).to(tdt)
    o = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), scale=0.125, causal=True, q_start=q_start)
    ro, *_ = OA.attention_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), scale=0.125, causal=True,
                              q_start=q_start)
    (assert_bf16 if dtype == "bf16" else assert_f32)(_np(o), ro)


@pytest.mark.parametrize("hq,hkv,chunks", [(4, 4, 3), (8, 2, 8), (2, 2, 1)])
def test_host_buffer_entry_point_matches_the_device_path(cuda, hq, hkv, chunks):
    import torch

    from pdum_dsl_b200 import kernels
    from pdum_dsl_b200.host import flash_attention_host

    g = torch.Generator(device="cpu").manual_seed(hq * 10 + chunks)
    q = torch.randn(2, hq, 300, 128, generator=g).to(torch.bfloat16).pin_memory()
    k = torch.randn(2, hkv, 300, 128, generator=g).to(torch.bfloat16).pin_memory()
    v = torch.randn(2, hkv, 300, 128, generator=g).to(torch.bfloat16).pin_memory()
    out = torch.empty_like(q).pin_memory()
    flash_attention_host(q, k, v, out, causal=True, chunks=chunks)
    want = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True).cpu()
    assert torch.equal(out, want)


def test_bf16_config4_gqa_slices(cuda):
    """Config 4 (B4 Hq64 Hkv8 S8192 D128 causal, GQA 8:1): full-size launch from seeded
    draws (seeds 40, 41, 42); 16 query heads covering every KV group vs the oracle."""
    import torch

    from pdum_dsl_b200 import kernels

    q = _seeded((4, 64, 8192, 128), 40, cuda)
    k = _seeded((4, 8, 8192, 128), 41, cuda)
    v = _seeded((4, 8, 8192, 128), 42, cuda)
    o = kernels.flash_attention(q, k, v, causal=True)
    kernels.check_device_errors()
    assert torch.isfinite(o).all()
    for b, h in [(b, 8 * g + (b + g) % 8) for b in range(4) for g in range(0, 8, 2)]:
        hk = h // 8
        ro, *_ = OA.attention_fwd(q[b, h].double().cpu().numpy(), k[b, hk].double().cpu().numpy(),
                                  v[b, hk].double().cpu().numpy(), scale=1 / math.sqrt(128), causal=True,
                                  row_block=1024)
        assert_bf16(_np(o[b, h]), ro, what=f"head ({b},{h})")


@pytest.mark.parametrize("D,DV,causal", [(96, 96, True), (128, 64, True), (64, 128, False), (80, 112, True),
                                         (72, 72, False), (32, 32, True), (16, 48, False), (56, 128, True),
                                         (256, 256, True), (192, 256, False), (136, 200, True), (256, 64, True),
                                         (64, 256, False)])
def test_bf16_head_dims_between_the_builds(cuda, D, DV, causal):
    """Head dims other than 64 / 128 / 256 (and e != o) on the tensor-core kernels: the
    tensor maps zero-fill the features up to the kernel's 64, 128 or 256."""
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(D * 3 + DV)
    q = torch.randn(1, 3, 300, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 3, 300, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 3, 300, DV, generator=g).to(torch.bfloat16)
    o = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), scale=1 / math.sqrt(D), causal=causal)
    kernels.check_device_errors()
    assert o.shape == (1, 3, 300, DV)
    ro, *_ = OA.attention_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), scale=1 / math.sqrt(D),
                              causal=causal)
    assert_bf16(_np(o), ro, what=f"D={D} DV={DV}")


def test_f32_head_dims_up_to_256(cuda):
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cpu").manual_seed(256)
    q, k = (torch.randn(1, 2, 150, 256, generator=g) for _ in range(2))
    v = torch.randn(1, 2, 150, 192, generator=g)
    o = kernels.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), scale=1 / 16, causal=True)
    ro, *_ = OA.attention_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), scale=1 / 16, causal=True)
    assert_f32(_np(o), ro)


@pytest.mark.parametrize("B,H,S,D", [(1, 32, 4096, 128), (1, 8, 1000, 64), (2, 3, 777, 96)])
def test_schedule_is_exact_under_sm_margin(cuda, B, H, S, D):
    """Small jobs deal their tiles heaviest first over the persistent grid; with
    SMs left free (sm_margin) the same tiles fall to other CTAs.  Every tile is
    computed the same way under either grid, so the outputs (and lse) are
    bit-identical, and every row is written (no tile lost or doubled)."""
    import torch

    from pdum_dsl_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(S + H)
    q, k, v = (torch.randn((B, H, S, D), device=cuda, generator=g).to(torch.bfloat16) for _ in range(3))
    o_dyn = torch.full_like(q, float("nan"))
    o_st = torch.full_like(q, float("nan"))
    for _ in range(3):  # repeated launches
        _, lse_dyn = kernels.flash_attention(q, k, v, causal=True, out=o_dyn, return_lse=True)
    _, lse_st = kernels.flash_attention(q, k, v, causal=True, out=o_st, return_lse=True, sm_margin=8)
    kernels.check_device_errors()
    assert torch.isfinite(o_dyn).all()
    assert torch.equal(o_dyn, o_st)
    assert torch.equal(lse_dyn, lse_st)
