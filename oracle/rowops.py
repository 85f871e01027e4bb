"""numpy f64 row softmax and two-pass layernorm -- test infrastructure (oracle).

Restates the reference's numpy denotations np_softmax and np_layernorm
(pdum/tl/zoo/zoo_common.py:33-35 and :69-72), which the reference's region
evaluator reproduces for the row-normalization / row-statistics regions
(zoo_common.py:56-60, :79-82; pinned by tests/golden fixtures).
"""

from __future__ import annotations

import numpy as np


def softmax(x, axis=-1):
    x = np.asarray(x, dtype=np.float64)
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


def layernorm(x, gamma=None, beta=None, eps=1e-5, axis=-1):
    x = np.asarray(x, dtype=np.float64)
    mu = x.mean(axis=axis, keepdims=True)
    xc = x - mu
    y = xc / np.sqrt((xc * xc).mean(axis=axis, keepdims=True) + eps)
    if gamma is not None:
        y = y * np.asarray(gamma, dtype=np.float64)
    if beta is not None:
        y = y + np.asarray(beta, dtype=np.float64)
    return y
