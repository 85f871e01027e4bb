"""The oracle pinned to the reference: numpy f64 restatements vs run_region fixtures."""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import rowops as OR
from tests.golden import HERE, input_checksum, load

ATTN = ["cfg1_flash_f32", "causal_bf16_ragged", "causal_bf16_d128", "noncausal_bf16_kv_ragged", "gqa_bf16",
        "causal_f32_small"]


def _gqa_flat(arr, spec_names):
    # (b, g, r, t, e) -> (b, g*r, t, e): query head h = g*r_count + r reads KV head g
    if "r" in spec_names:
        b, g, r = arr.shape[:3]
        return arr.reshape(b, g * r, *arr.shape[3:])
    return arr


@pytest.mark.parametrize("case", ATTN)
def test_inputs_regenerate_exactly(case):
    spec, ins, _ = load(case)
    for s, a in zip(spec["inputs"], ins):
        assert input_checksum(a) == s["checksum"]


@pytest.mark.parametrize("case", ATTN)
def test_attention_oracle_matches_run_region(case):
    spec, (q, k, v), outs = load(case)
    kw = spec["region"]
    qn = spec["inputs"][0]["names"]
    q4 = _gqa_flat(q, qn)
    o, m, den, _ = OA.attention_fwd(q4, k, v, scale=kw.get("scale"), causal=kw["causal"])
    o = o.reshape(outs[0].shape)
    np.testing.assert_allclose(o, outs[0], rtol=1e-11, atol=1e-12)
    if kw.get("artifacts"):
        np.testing.assert_allclose(m.reshape(outs[1].shape), outs[1], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(den.reshape(outs[2].shape), outs[2], rtol=1e-11, atol=1e-12)


def test_flash_tile_flagship():
    z = np.load(HERE / "flash_tile_default.npz")
    o, *_ = OA.attention_fwd(z["q"], z["k"], z["v"], causal=True)
    np.testing.assert_allclose(o, z["naive"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(o, z["tile"], rtol=1e-12, atol=1e-14)  # the planned online-softmax kernel
    np.testing.assert_allclose(o, z["oracle"], rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("case", ["flash_joint_bwd", "flash_joint_bwd_d64"])
def test_backward_oracle_matches_autodiff_joint(case):
    spec, (q, k, v, dout), (out, dq, dk, dv) = load(case)
    assert spec["outputs"][0] == "out"
    o, *_ = OA.attention_fwd(q, k, v, causal=True)
    gq, gk, gv = OA.attention_bwd(q, k, v, dout, causal=True)
    np.testing.assert_allclose(o, out, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(gq, dq, rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(gk, dk, rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(gv.T, dv, rtol=1e-9, atol=1e-10)  # the joint yields dv as (o, s)


@pytest.mark.parametrize("case", ["rowsoftmax_16x4096", "rowsoftmax_37x1001"])
def test_softmax_oracle(case):
    _, (x,), (y,) = load(case)
    np.testing.assert_allclose(OR.softmax(x), y, rtol=1e-13, atol=1e-16)


@pytest.mark.parametrize("case", ["layernorm_16x4096", "layernorm_37x1001"])
def test_layernorm_oracle(case):
    spec, (x, g, b), (y,) = load(case)
    np.testing.assert_allclose(OR.layernorm(x, g, b, spec["region"]["eps"]), y, rtol=1e-12, atol=1e-12)


def test_bwd_oracle_is_the_gradient():
    """finite-difference check of the closed-form adjoint (scaled, GQA, causal)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 4, 7, 5))
    k = rng.standard_normal((1, 2, 7, 5))
    v = rng.standard_normal((1, 2, 7, 3))
    w = rng.standard_normal((1, 4, 7, 3))
    f = lambda q_, k_, v_: (OA.attention_fwd(q_, k_, v_, scale=0.7, causal=True)[0] * w).sum()
    dq, dk, dv = OA.attention_bwd(q, k, v, w, scale=0.7, causal=True)
    eps = 1e-6
    for arr, g in ((q, dq), (k, dk), (v, dv)):
        idx = (0, 1, 3, 2)
        a1, a2 = arr.copy(), arr.copy()
        a1[idx] += eps
        a2[idx] -= eps
        args1 = [a1 if x is arr else x for x in (q, k, v)]
        args2 = [a2 if x is arr else x for x in (q, k, v)]
        fd = (f(*args1) - f(*args2)) / (2 * eps)
        assert abs(fd - g[idx]) < 1e-6
