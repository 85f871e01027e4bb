"""numpy f64 attention forward / backward -- test infrastructure (oracle).

Forward: the reference's numpy denotation of attention
(pdum/tl/zoo/tiles.py:254-257, pdum/tl/zoo/attention.py:191-194):
``softmax(where(mask, scale * q k^T, -1e9), axis=s) @ v`` with the causal mask
``s <= t`` in absolute coordinates (dialect.py:1382-1383), extended with the
rider dims (batch, head) and GQA head groups that the widened flash rows take
(query head h reads KV head h // group, pdum/tl/zoo/llama.py:7-8,51-54).
The artifact finals are m = max_s score and den = sum_s exp(score - m)
(fusion.py:611-613); lse = m + log(den).

Backward: the adjoint that autodiff.grad derives for the naive region
(autodiff.py:102-150), in closed form: P = softmax(...), dV = P^T dO,
dP = dO V^T, dS = P * (dP - rowsum(dP * P)) (the D-class identity pinned by
conformance/test_fusion_triton.py:195-220), dQ = scale dS K, dK = scale dS^T Q;
GQA sums dK/dV over the query heads of a group.  Masked scores carry zero
gradient (where's adjoint routes dS only through the kept branch).

Work is chunked over (batch, head) and query-row slabs so full-size heads fit
in memory; numpy's matmul (BLAS, multi-threaded) does the contractions.
"""

from __future__ import annotations

import numpy as np

FILL = -1e9  # the reference's mask fill (zoo_common.py:86, tiles.py:223)


def _as4(x):
    x = np.asarray(x, dtype=np.float64)
    while x.ndim < 4:
        x = x[None]
    return x


def _scores(qh, kh, scale, causal, t0, q_start):
    sc = qh @ kh.T
    if scale is not None:
        sc = sc * scale
    if causal:
        t = np.arange(t0, t0 + qh.shape[0])[:, None] + q_start
        s = np.arange(kh.shape[0])[None, :]
        sc = np.where(s <= t, sc, FILL)
    return sc


def attention_fwd(q, k, v, *, scale=None, causal=False, q_start=0, row_block=1024):
    """Returns (o, m, den, lse); shapes follow q's leading dims."""
    lead = np.shape(q)[:-1]
    q4, k4, v4 = _as4(q), _as4(k), _as4(v)
    B, H, T, _ = q4.shape
    HKV = k4.shape[1]
    group = H // HKV
    DV = v4.shape[3]
    o = np.empty((B, H, T, DV))
    m = np.empty((B, H, T))
    den = np.empty((B, H, T))
    for b in range(B):
        for h in range(H):
            kh, vh = k4[b, h // group], v4[b, h // group]
            for t0 in range(0, T, row_block):
                sc = _scores(q4[b, h, t0:t0 + row_block], kh, scale, causal, t0, q_start)
                mx = sc.max(axis=1, keepdims=True)
                e = np.exp(sc - mx)
                dn = e.sum(axis=1, keepdims=True)
                o[b, h, t0:t0 + row_block] = (e / dn) @ vh
                m[b, h, t0:t0 + row_block] = mx[:, 0]
                den[b, h, t0:t0 + row_block] = dn[:, 0]
    lse = m + np.log(den)
    return (o.reshape(*lead, DV), m.reshape(lead), den.reshape(lead), lse.reshape(lead))


def attention_bwd(q, k, v, dout, *, scale=None, causal=False, q_start=0, row_block=1024):
    """Returns (dq, dk, dv) for out = attention(q, k, v), upstream dout."""
    shapes = (np.shape(q), np.shape(k), np.shape(v))
    q4, k4, v4, do4 = _as4(q), _as4(k), _as4(v), _as4(dout)
    B, H, T, _ = q4.shape
    HKV = k4.shape[1]
    group = H // HKV
    sc_mul = 1.0 if scale is None else scale
    dq = np.zeros_like(q4)
    dk = np.zeros_like(k4)
    dv = np.zeros_like(v4)
    for b in range(B):
        for h in range(H):
            hk = h // group
            kh, vh = k4[b, hk], v4[b, hk]
            for t0 in range(0, T, row_block):
                qh = q4[b, h, t0:t0 + row_block]
                doh = do4[b, h, t0:t0 + row_block]
                sc = _scores(qh, kh, scale, causal, t0, q_start)
                e = np.exp(sc - sc.max(axis=1, keepdims=True))
                P = e / e.sum(axis=1, keepdims=True)
                dv[b, hk] += P.T @ doh
                dP = doh @ vh.T
                dS = P * (dP - (dP * P).sum(axis=1, keepdims=True))
                if causal:
                    t = np.arange(t0, t0 + qh.shape[0])[:, None] + q_start
                    dS = np.where(np.arange(kh.shape[0])[None, :] <= t, dS, 0.0)
                dq[b, h, t0:t0 + row_block] = sc_mul * (dS @ kh)
                dk[b, hk] += sc_mul * (dS.T @ qh)
    return dq.reshape(shapes[0]), dk.reshape(shapes[1]), dv.reshape(shapes[2])


def masked_attention(q, k, v, visible, *, scale=None):
    """One head under an arbitrary boolean mask ``visible`` (t, s): the reference's
    denotation ``softmax(where(mask, scale * q k^T, -1e9)) @ v`` (zoo/attention.py:
    98-101 spells the sliding window this way)."""
    sc = np.asarray(q, dtype=np.float64) @ np.asarray(k, dtype=np.float64).T
    if scale is not None:
        sc = sc * scale
    sc = np.where(visible, sc, FILL)
    p = np.exp(sc - sc.max(axis=1, keepdims=True))
    return (p / p.sum(axis=1, keepdims=True)) @ np.asarray(v, dtype=np.float64)
