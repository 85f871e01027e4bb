"""Device-tensor entry points over the C ABI (the zero-copy fast path).

Each function takes CUDA tensors, fills a descriptor of ``include/pdb.h`` and
launches on the current torch stream.  Nothing here computes on the host and
nothing falls back: a CPU tensor, a dtype the library does not build, or a
missing ``libpdb_sm100.so`` raises.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import _lib
from ._lib import FlashBwdDesc, FlashDesc, LayerNormDesc, RowSoftmaxDesc, check, load

_DTYPES = {torch.float32: _lib.PDB_F32, torch.bfloat16: _lib.PDB_BF16}


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("pdum_dsl_b200 kernels take CUDA tensors (no host fallback)")


def _rows2d(x: torch.Tensor) -> torch.Tensor:
    if x.dim() < 1 or x.stride(-1) != 1:
        x = x.contiguous()
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.dim() == 2 and x2.shape[0] > 0 and x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def row_softmax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax over the last dim of an f32 CUDA tensor (row-normalization)."""
    _need_cuda(x)
    if x.dtype != torch.float32:
        raise TypeError("row_softmax: float32 only")
    x2 = _rows2d(x)
    y = torch.empty_like(x2) if out is None else out.view(x2.shape)
    d = RowSoftmaxDesc(x2.data_ptr(), y.data_ptr(), x2.shape[0], x2.shape[1], x2.stride(0) if x2.shape[0] else
                       x2.shape[1], y.stride(0) if y.shape[0] else y.shape[1])
    check(load().pdb_rowsoftmax_f32(C.byref(d), _stream(x)), "pdb_rowsoftmax_f32")
    return y.view(x.shape)


def layernorm(x: torch.Tensor, gamma: torch.Tensor | None = None, beta: torch.Tensor | None = None,
              eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
    """Two-pass layernorm over the last dim (row-statistics), f32."""
    _need_cuda(x)
    if x.dtype != torch.float32:
        raise TypeError("layernorm: float32 only")
    x2 = _rows2d(x)
    C_ = x2.shape[1]
    for nm, t in (("gamma", gamma), ("beta", beta)):
        if t is not None and (t.dtype != torch.float32 or t.numel() != C_ or not t.is_cuda):
            raise ValueError(f"layernorm: {nm} must be a CUDA f32 vector of length {C_}")
    g = gamma.contiguous() if gamma is not None else None
    b = beta.contiguous() if beta is not None else None
    y = torch.empty_like(x2) if out is None else out.view(x2.shape)
    d = LayerNormDesc(x2.data_ptr(), g.data_ptr() if g is not None else None, b.data_ptr() if b is not None else None,
                      y.data_ptr(), x2.shape[0], C_, x2.stride(0) if x2.shape[0] else C_,
                      y.stride(0) if y.shape[0] else C_, float(eps))
    check(load().pdb_layernorm_f32(C.byref(d), _stream(x)), "pdb_layernorm_f32")
    return y.view(x.shape)


def _as4d(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() == 2:
        t = t[None, None]
    elif t.dim() == 3:
        t = t[None]
    elif t.dim() != 4:
        raise ValueError(f"{name}: expected (T, D), (H, T, D) or (B, H, T, D), got {tuple(t.shape)}")
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _s3(t: torch.Tensor):
    return _lib.I64x3(t.stride(0), t.stride(1), t.stride(2))


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float | None = None,
                    causal: bool = False, q_start: int = 0, out: torch.Tensor | None = None,
                    return_lse: bool = False, return_artifacts: bool = False, key_intervals=None,
                    sm_margin: int = 0):
    """softmax(scale * q k^T [causal: s <= t + q_start]) v.

    q (B, Hq, T, D), k/v (B, Hkv, S, D|Dv) with Hq a multiple of Hkv (GQA);
    2-D and 3-D inputs drop the leading dims.  bf16 runs the tcgen05 kernel
    (D, Dv multiples of 8 up to 256); f32 runs the IEEE CUDA-core kernel (any D, Dv <= 256).  Returns o, or
    (o, lse) / (o, m, den) with the per-row float32 statistics.
    ``key_intervals`` (a ``recognize.KeyIntervals`` of T rows) is a general
    closed mask: row t sees keys lo[t] <= s < hi[t] (``causal`` must be False).
    ``sm_margin`` SMs are left free by the persistent bf16 grid (for a collective
    that runs alongside, e.g. the all-gather of the previous slab's output)."""
    _need_cuda(q, k, v)
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"flash_attention: q/k/v must share dtype float32 or bfloat16, got {q.dtype}/{k.dtype}/{v.dtype}")
    shape_in = q.shape
    q4, k4, v4 = _as4d(q, "q"), _as4d(k, "k"), _as4d(v, "v")
    B, H, T, D = q4.shape
    Bk, HKV, S, Dk = k4.shape
    if Bk != B or Dk != D or v4.shape[:3] != (B, HKV, S):
        raise ValueError(f"flash_attention: incompatible q {tuple(q4.shape)} k {tuple(k4.shape)} v {tuple(v4.shape)}")
    DV = v4.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty((B, H, T, DV), dtype=q.dtype, device=q.device) if out is None else _as4d(out, "out")
    stats = {}
    want = ("lse",) if return_lse else ()
    want += ("m", "den") if return_artifacts else ()
    for nm in want:
        stats[nm] = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    d = FlashDesc()
    d.q, d.k, d.v, d.o = q4.data_ptr(), k4.data_ptr(), v4.data_ptr(), o.data_ptr()
    d.lse = stats["lse"].data_ptr() if "lse" in stats else None
    d.m = stats["m"].data_ptr() if "m" in stats else None
    d.den = stats["den"].data_ptr() if "den" in stats else None
    d.batch, d.heads_q, d.heads_kv, d.seqlen_q, d.seqlen_k, d.head_dim, d.head_dim_v = B, H, HKV, T, S, D, DV
    d.q_stride, d.k_stride, d.v_stride, d.o_stride = _s3(q4), _s3(k4), _s3(v4), _s3(o)
    d.q_start, d.scale, d.causal, d.dtype = int(q_start), float(scale), int(bool(causal)), _DTYPES[q.dtype]
    d.sm_margin = int(sm_margin)
    keep = None
    if key_intervals is not None:
        if causal:
            raise ValueError("flash_attention: key_intervals replace the causal flag")
        if len(key_intervals.lo) != T:
            raise ValueError(f"flash_attention: key_intervals has {len(key_intervals.lo)} rows, q has {T}")
        keep = torch.from_numpy(np.stack([key_intervals.lo, key_intervals.hi])).to(q.device)
        d.key_lo, d.key_hi = keep[0].data_ptr(), keep[1].data_ptr()
        d.mask_monotone = int(key_intervals.monotone)
    check(load().pdb_flash_fwd(C.byref(d), _stream(q)), "pdb_flash_fwd")
    del keep  # the launch is stream-ordered before any reuse of this memory by the caching allocator
    o_ret = o.view(*shape_in[:-1], DV) if out is None else out
    lead = shape_in[:-1]
    if return_artifacts:
        extra = (stats["lse"].view(lead),) if return_lse else ()
        return (o_ret, *extra, stats["m"].view(lead), stats["den"].view(lead))
    if return_lse:
        return o_ret, stats["lse"].view(lead)
    return o_ret


def flash_attention_backward(q, k, v, o, dout, lse=None, *, scale=None, causal=False, q_start=0):
    """(dq, dk, dv) of flash_attention; ``lse`` None recomputes it."""
    _need_cuda(q, k, v, o, dout)
    if q.dtype not in _DTYPES:
        raise TypeError("flash_attention_backward: float32 or bfloat16")
    shape_q, shape_k, shape_v = q.shape, k.shape, v.shape
    q4, k4, v4, o4, do4 = (_as4d(t, n) for t, n in ((q, "q"), (k, "k"), (v, "v"), (o, "o"), (dout, "dout")))
    B, H, T, D = q4.shape
    _, HKV, S, _ = k4.shape
    DV = v4.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dq, dk, dv = torch.empty_like(q4), torch.empty_like(k4), torch.empty_like(v4)
    d = FlashBwdDesc()
    d.q, d.k, d.v, d.o, d.dout = q4.data_ptr(), k4.data_ptr(), v4.data_ptr(), o4.data_ptr(), do4.data_ptr()
    lse_c = lse.contiguous().view(B, H, T) if lse is not None else None
    d.lse = lse_c.data_ptr() if lse_c is not None else None
    d.dq, d.dk, d.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    d.batch, d.heads_q, d.heads_kv, d.seqlen_q, d.seqlen_k, d.head_dim, d.head_dim_v = B, H, HKV, T, S, D, DV
    d.q_stride, d.k_stride, d.v_stride, d.o_stride, d.do_stride = _s3(q4), _s3(k4), _s3(v4), _s3(o4), _s3(do4)
    d.dq_stride, d.dk_stride, d.dv_stride = _s3(dq), _s3(dk), _s3(dv)
    d.q_start, d.scale, d.causal, d.dtype = int(q_start), float(scale), int(bool(causal)), _DTYPES[q.dtype]
    lib = load()
    nbytes = lib.pdb_flash_bwd_workspace_size(C.byref(d))
    ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=q.device)
    d.workspace, d.workspace_bytes = ws.data_ptr(), int(nbytes)
    check(lib.pdb_flash_bwd(C.byref(d), _stream(q)), "pdb_flash_bwd")
    return dq.view(shape_q), dk.view(shape_k), dv.view(shape_v)


def check_device_errors() -> None:
    """Synchronise the current stream and raise if a bounded device wait expired."""
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(load().pdb_check_error(s), "pdb_check_error")


def _ew_program(ops, out_shape):
    """ops: list of (name, operand) with operand None (unary), a float, or a CUDA
    float32 tensor broadcastable to out_shape (batch, m, n)."""
    if len(ops) > _lib.MAX_EW_OPS:
        raise ValueError(f"at most {_lib.MAX_EW_OPS} epilogue steps")
    arr = (_lib.EwOp * _lib.MAX_EW_OPS)()
    keep = []
    for i, (name, operand, swap) in enumerate(ops):
        o = arr[i]
        o.op = _lib.EW_OPS[name]
        o.swap = int(bool(swap))
        if operand is None:
            o.operand = 0
        elif isinstance(operand, (int, float)):
            o.operand, o.value = 1, float(operand)
        else:
            t = operand.float().expand(out_shape)
            keep.append(t)
            o.operand, o.ptr = 2, t.data_ptr()
            o.stride = _lib.I64x3(t.stride(0), t.stride(1), t.stride(2))
    return arr, keep


def contract(a: torch.Tensor, b: torch.Tensor, *, epilogue=(), alpha: float = 1.0,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """c[b, m, n] = epilogue(alpha * sum_k a[b, m, k] * b[b, n, k]).

    a (batch, m, k), b (batch, n, k): f32 (IEEE path, f32 out) or bf16 with k
    contiguous (tcgen05 path, bf16 out).  ``epilogue`` is a sequence of
    (op, operand, swap) steps with operand None (unary), a float, or a CUDA
    tensor broadcastable to (batch, m, n)."""
    _need_cuda(a, b)
    if a.dtype not in _DTYPES or b.dtype != a.dtype:
        raise TypeError("contract: a and b must both be float32 or bfloat16")
    Bt, M, K = a.shape
    Bb, N, Kb = b.shape
    if Bb != Bt or Kb != K:
        raise ValueError(f"contract: incompatible a {tuple(a.shape)} b {tuple(b.shape)}")
    if a.dtype == torch.bfloat16:
        a = a if a.stride(2) == 1 else a.contiguous()
        b = b if b.stride(2) == 1 else b.contiguous()
    c = torch.empty((Bt, M, N), dtype=a.dtype, device=a.device) if out is None else out
    d = _lib.ContractDesc()
    d.a, d.b, d.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.batch, d.m, d.n, d.k = Bt, M, N, K
    d.a_stride, d.b_stride, d.c_stride = _s3(a), _s3(b), _s3(c)
    d.alpha, d.dtype = float(alpha), _DTYPES[a.dtype]
    ops, keep = _ew_program(list(epilogue), (Bt, M, N))
    d.ops, d.n_ops = ops, len(epilogue)
    check(load().pdb_contract(C.byref(d), _stream(a)), "pdb_contract")
    del keep
    return c


def pointwise(x: torch.Tensor, program, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = program(x) elementwise over an f32 (batch, m, n) CUDA tensor (map-chain)."""
    _need_cuda(x)
    if x.dtype != torch.float32 or x.dim() != 3:
        raise TypeError("pointwise: a 3-D float32 tensor")
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device) if out is None else out
    d = _lib.PointwiseDesc()
    d.x, d.y = x.data_ptr(), y.data_ptr()
    d.batch, d.m, d.n = x.shape
    d.x_stride, d.y_stride = _s3(x), _s3(y)
    ops, keep = _ew_program(list(program), tuple(x.shape))
    d.ops, d.n_ops = ops, len(program)
    check(load().pdb_pointwise_f32(C.byref(d), _stream(x)), "pdb_pointwise_f32")
    del keep
    return y
