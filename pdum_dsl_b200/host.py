"""Host-buffer entry point: flash attention on pinned host tensors, pipelined.

The reference's lowering (``conformance/triton_tile.py:676-698``) copies its
numpy inputs to the device, launches, synchronises and copies the output back,
one step after the other.  ``flash_attention_host`` does the same job for
host-resident q / k / v / out, but splits the (batch, KV-head) units into
chunks and runs three CUDA streams -- host-to-device copies, the sm_100a
kernel, device-to-host copies -- so the PCIe traffic of one chunk overlaps the
compute of the next and both copy directions run at once.  Device staging
buffers are allocated per call (two chunks deep) through torch's caching
allocator.  Host tensors may be float32 / float64 (the reference's numpy
convention) while the kernel runs bf16: each chunk is copied in its host dtype
and cast on the device, and the output is cast back before its copy out.
"""

from __future__ import annotations

import math

import torch

from . import kernels


def flash_attention_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *,
                         scale: float | None = None, causal: bool = False, chunks: int = 8,
                         device: torch.device | None = None, compute_dtype: torch.dtype | None = None,
                         q_start: int = 0, key_intervals=None) -> torch.Tensor:
    """q (B, Hq, T, D), k / v (B, Hkv, S, D), out (B, Hq, T, Dv): contiguous host
    tensors (pin them for full PCIe speed).  ``compute_dtype`` (default: q's
    dtype) is what the kernel runs in.  Returns ``out`` after the device work has
    completed."""
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.is_cuda or not t.is_contiguous() or t.dim() != 4:
            raise ValueError(f"{name}: expected a contiguous 4-D host tensor")
    dev = device or torch.device("cuda", torch.cuda.current_device())
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv:
        raise ValueError("heads_q must be a multiple of heads_kv")
    r = Hq // Hkv
    units = B * Hkv
    qf = q.view(units, r, T, D)
    kf, vf = k.view(units, 1, *k.shape[2:]), v.view(units, 1, *v.shape[2:])
    of = out.view(units, r, T, out.shape[3])
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    n = max(1, min(chunks, units))
    bounds = [(units * i // n, units * (i + 1) // n) for i in range(n)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    cur = torch.cuda.current_stream(dev)
    for s in (s_in, s_cmp, s_out):
        s.wait_stream(cur)
    depth = 2
    size = max(hi - lo for lo, hi in bounds)
    cdt = compute_dtype or q.dtype
    cast = any(t.dtype != cdt for t in (q, k, v, out))
    bufs = [{name: torch.empty((size,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
             for name, t in (("q", qf), ("k", kf), ("v", vf), ("o", of))} for _ in range(depth)]
    if cast:  # device-side casts between the host dtype and the compute dtype
        for b in bufs:
            for name in ("q", "k", "v", "o"):
                b["c" + name] = torch.empty(b[name].shape, dtype=cdt, device=dev)
    loaded = [torch.cuda.Event() for _ in range(n)]
    computed = [torch.cuda.Event() for _ in range(n)]
    drained = [torch.cuda.Event() for _ in range(n)]
    for i, (lo, hi) in enumerate(bounds):
        b = bufs[i % depth]
        m = hi - lo
        with torch.cuda.stream(s_in):
            if i >= depth:
                s_in.wait_event(computed[i - depth])  # inputs of this slot no longer read
            for name, src in (("q", qf), ("k", kf), ("v", vf)):
                b[name][:m].copy_(src[lo:hi], non_blocking=True)
            loaded[i].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(loaded[i])
            if i >= depth:
                s_cmp.wait_event(drained[i - depth])  # output of this slot copied out
            src = {}
            for name in ("q", "k", "v"):
                if cast:
                    b["c" + name][:m].copy_(b[name][:m])
                src[name] = b[("c" if cast else "") + name][:m]
            ob = b["co" if cast else "o"][:m]
            qj = src["q"].reshape(1, m * r, T, D)
            kj = src["k"].reshape(1, m, *kf.shape[2:])
            vj = src["v"].reshape(1, m, *vf.shape[2:])
            kernels.flash_attention(qj, kj, vj, scale=scale, causal=causal, q_start=q_start,
                                    key_intervals=key_intervals, out=ob.reshape(1, m * r, T, of.shape[3]))
            if cast:
                b["o"][:m].copy_(ob)
            computed[i].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(computed[i])
            of[lo:hi].copy_(b["o"][:m], non_blocking=True)
            drained[i].record(s_out)
    cur.wait_stream(s_out)
    torch.cuda.current_stream(dev).synchronize()
    return out
