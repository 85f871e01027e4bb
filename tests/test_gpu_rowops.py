"""Row softmax / layernorm kernels vs the reference's run_region fixtures and the oracle."""

import numpy as np
import pytest

from oracle import rowops as OR
from tests.golden import load
from tests.tolerances import assert_f32

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32), device=dev)


@pytest.mark.parametrize("case", ["rowsoftmax_16x4096", "rowsoftmax_37x1001"])
def test_row_softmax_matches_reference(cuda, case):
    from pdum_dsl_b200 import kernels

    _, (x,), (y,) = load(case)
    got = kernels.row_softmax(_t(x, cuda)).cpu().numpy()
    assert_f32(got, y, what=case)


@pytest.mark.parametrize("case", ["layernorm_16x4096", "layernorm_37x1001"])
def test_layernorm_matches_reference(cuda, case):
    from pdum_dsl_b200 import kernels

    spec, (x, g, b), (y,) = load(case)
    got = kernels.layernorm(_t(x, cuda), _t(g, cuda), _t(b, cuda), eps=spec["region"]["eps"]).cpu().numpy()
    assert_f32(got, y, what=case)


@pytest.mark.parametrize("R,C", [(1, 1), (3, 4), (5, 7), (2, 8192), (3, 8196), (2, 20000), (0, 16)])
def test_row_shapes_and_ragged(cuda, R, C):
    from pdum_dsl_b200 import kernels

    rng = np.random.default_rng(R * 131 + C)
    x = rng.standard_normal((R, C)).astype(np.float32) * 3
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    xs = _t(x, cuda)
    ys = kernels.row_softmax(xs).cpu().numpy()
    yl = kernels.layernorm(xs, _t(g, cuda), _t(b, cuda)).cpu().numpy()
    if R:
        assert_f32(ys, OR.softmax(x.astype(np.float64)), what="softmax")
        assert_f32(yl, OR.layernorm(x.astype(np.float64), g, b), what="layernorm")


def test_strided_rows_and_large_magnitudes(cuda):
    import torch

    from pdum_dsl_b200 import kernels

    rng = np.random.default_rng(3)
    base = (rng.standard_normal((64, 4100)) * 40).astype(np.float32)  # wide scores: exp near saturation
    xt = _t(base, cuda)[:, :4096]  # row stride 4100 (not 16-byte aligned rows -> generic path)
    assert_f32(kernels.row_softmax(xt).cpu().numpy(), OR.softmax(base[:, :4096].astype(np.float64)))
    x2 = _t(base, cuda)[:, 4:4100]  # aligned? 4 floats = 16 B offset, stride 4100 -> not multiple of 4
    assert_f32(kernels.layernorm(x2).cpu().numpy(), OR.layernorm(base[:, 4:4100].astype(np.float64)))
    out = torch.empty(64, 4096, device=cuda)
    kernels.row_softmax(xt, out=out)
    assert_f32(out.cpu().numpy(), OR.softmax(base[:, :4096].astype(np.float64)))


def test_full_config_properties(cuda):
    """Config 2 (X 8192 x 4096 ~ N(0,1), gamma ~ N(1, 0.1), beta ~ N(0, 0.1), eps 1e-5, seeds
    20..22): size-independent properties over every row, plus sampled rows vs the oracle."""
    import torch

    from pdum_dsl_b200 import kernels

    rng = [np.random.default_rng(20 + i) for i in range(3)]
    xh = rng[0].standard_normal((8192, 4096), dtype=np.float32)
    gam = (1 + 0.1 * rng[1].standard_normal(4096)).astype(np.float32)
    bet = (0.1 * rng[2].standard_normal(4096)).astype(np.float32)
    x = torch.from_numpy(xh).to(cuda)
    y = kernels.row_softmax(x)
    sums = y.double().sum(dim=1)
    assert torch.allclose(sums, torch.ones_like(sums), atol=1e-5)
    assert (y >= 0).all()
    idx = [0, 1, 777, 4095, 5000, 8191]
    assert_f32(y[idx].cpu().numpy(), OR.softmax(xh[idx].astype(np.float64)))
    g, b = torch.from_numpy(gam).to(cuda), torch.from_numpy(bet).to(cuda)
    ln = kernels.layernorm(x, g, b, eps=1e-5)
    # undo the affine epilogue: the normalised rows have mean 0 and variance 1
    z = (ln.double() - b.double()) / g.double()
    assert torch.allclose(z.mean(1), torch.zeros(8192, dtype=torch.float64, device=cuda), atol=1e-4)
    assert torch.allclose(z.var(1, unbiased=False), torch.ones(8192, dtype=torch.float64, device=cuda), atol=1e-3)
    assert_f32(ln[idx].cpu().numpy(), OR.layernorm(xh[idx].astype(np.float64), gam.astype(np.float64),
                                                  bet.astype(np.float64), eps=1e-5))
