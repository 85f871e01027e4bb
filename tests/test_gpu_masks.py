"""General closed masks (sliding window, block-diagonal, the zoo's sliding_attention)
through the drop-in lowering, f32 and bf16, vs the reference's run_region fixtures."""

import numpy as np
import pytest

from tests.golden import load
from tests.tolerances import assert_bf16, assert_f32

pytestmark = pytest.mark.gpu

CASES = ["sliding_zoo_f32", "sliding_zoo_bf16", "sliding_bf16_riders", "block_bf16_d128", "block_causal_f32"]


def _region(kw):
    if kw.get("zoo") == "sliding_attention":
        from pdum.tl.zoo.attention import sliding_attention

        return sliding_attention(**{k: v for k, v in kw.items() if k != "zoo"}).region
    from pdum_dsl_b200.regions import attention_region

    return attention_region(**kw)


@pytest.mark.parametrize("case", CASES)
def test_masked_flash_matches_run_region(cuda, dsl, case):
    from pdum_dsl_b200.plan import plan_region
    from pdum_dsl_b200.tile import compile_tile

    spec, ins, (want,) = load(case)
    region = _region(spec["region"])
    dtype = spec["inputs"][0]["dtype"]
    (g,) = plan_region(region).groups
    assert g.template == "flash"
    run = compile_tile(g.kernel, dtype=dtype)
    assert run.spec.mask is not None and not run.spec.causal
    got = run(ins)
    (assert_bf16 if dtype == "bf16" else assert_f32)(got, want, what=case)


@pytest.mark.parametrize("dtype,D", [("f32", 64), ("bf16", 64), ("bf16", 128), ("bf16", 256)])
def test_sliding_window_long_rows_vs_oracle(cuda, dsl, dtype, D):
    """A longer sliding window (S=2000, W=300, two heads): the kernels visit only each
    block's live key tiles, and the rows of a block whose window starts past the block's
    first key tiles see only masked scores there; checked against the oracle."""
    import torch

    from oracle import attention as OA
    from pdum_dsl_b200.regions import attention_region
    from pdum_dsl_b200.tile import compile_tile

    T, W = 2000, 300
    region = attention_region(H=2, T=T, D=D, causal=True, window=W, scale=0.125)
    run = compile_tile(region, dtype=dtype)
    assert run.spec.mask.monotone
    rng = np.random.default_rng(77)
    q, k, v = (rng.standard_normal((2, T, D)).astype(np.float32) for _ in range(3))
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    tq, tk, tv = (torch.from_numpy(x).cuda().to(dt) for x in (q, k, v))
    got = run.run_t(tq, tk, tv).float().cpu().numpy()
    qq, kk, vv = (x.float().cpu().numpy().astype(np.float64) for x in (tq, tk, tv))
    t = np.arange(T)[:, None]
    s = np.arange(T)[None, :]
    visible = (s <= t) & (t - s < W)
    want = np.stack([OA.masked_attention(qq[h], kk[h], vv[h], visible, scale=0.125) for h in range(2)])
    (assert_bf16 if dtype == "bf16" else assert_f32)(got, want)
