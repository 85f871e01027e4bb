"""The parity bars of the hot path (from the project's north star).

* f32 results: within 1e-5 relative error of the reference's f64 evaluation,
  measured as max|got - ref| <= 1e-5 * max|ref| over the output tensor.
* bf16 (fp32-accumulate) results: within 2e-2 absolute error of the
  reference evaluation on the same bf16-rounded inputs.
"""

import numpy as np

F32_REL = 1e-5
BF16_ABS = 2e-2


def assert_f32(got, ref, rel=F32_REL, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = np.abs(got - ref).max()
    bound = rel * max(np.abs(ref).max(), 1e-30)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err <= bound, f"{what}: max abs err {err:.3e} > {rel} * max|ref| = {bound:.3e}"


def assert_bf16(got, ref, atol=BF16_ABS, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref).max()
    assert err <= atol, f"{what}: max abs err {err:.3e} > {atol}"
