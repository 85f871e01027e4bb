"""pdb_flash_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers own no allocator at call time -- a memory pool or arena that has
claimed the whole device, or a plain C host with no allocator binding -- so
they cannot provide pdb_flash_bwd's workspace.  The no-alloc entry point uses
a fixed scratch array inside the library instead.  These tests call it through
the C ABI twice in a row (the scratch keeps the previous call's contents) and
compare with pdb_flash_bwd given a caller workspace, at the bf16 tolerance.
This file is collected last on purpose.
"""

import ctypes as C
import math

import pytest

from tests.tolerances import BF16_ABS

pytestmark = pytest.mark.gpu


def _desc(q, k, v, o, do, lse, dq, dk, dv, scale, causal):
    from pdum_dsl_b200 import _lib

    s3 = lambda t: _lib.I64x3(t.stride(0), t.stride(1), t.stride(2))
    d = _lib.FlashBwdDesc()
    d.q, d.k, d.v, d.o, d.dout = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr()
    d.lse = lse.data_ptr() if lse is not None else None
    d.dq, d.dk, d.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    B, H, T, D = q.shape
    d.batch, d.heads_q, d.heads_kv, d.seqlen_q, d.seqlen_k = B, H, k.shape[1], T, k.shape[2]
    d.head_dim, d.head_dim_v = D, v.shape[3]
    d.q_stride, d.k_stride, d.v_stride, d.o_stride, d.do_stride = s3(q), s3(k), s3(v), s3(o), s3(do)
    d.dq_stride, d.dk_stride, d.dv_stride = s3(dq), s3(dk), s3(dv)
    d.scale, d.causal, d.dtype = scale, int(causal), _lib.PDB_BF16
    return d


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("stored_lse", [True, False])
def test_noalloc_matches_workspace_backward_twice(cuda, stored_lse, D):
    """head_dim 64 runs the fused single pass (its fp32 dQ accumulator lives in the
    scratch); head_dim 128 the dK/dV and dQ kernels sharing the scratch's two
    work-unit counters -- both back to back, with the previous call's leftovers."""
    import torch

    from pdum_dsl_b200 import _lib, kernels

    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (B, H, HKV, T) in enumerate(((2, 4, 2, 300), (1, 2, 2, 513))):  # two calls, different sizes
        g = torch.Generator(device="cpu").manual_seed(100 + call)
        q = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(cuda)
        k, v = (torch.randn(B, HKV, T, D, generator=g).to(torch.bfloat16).to(cuda) for _ in range(2))
        do = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(cuda)
        scale = 1 / math.sqrt(D)
        o, lse = kernels.flash_attention(q, k, v, scale=scale, causal=True, return_lse=True)
        ref = kernels.flash_attention_backward(q, k, v, o, do, lse if stored_lse else None, scale=scale, causal=True)
        got = [torch.empty_like(x) for x in (q, k, v)]
        d = _desc(q, k, v, o, do, lse if stored_lse else None, *got, scale, True)
        assert lib.pdb_flash_bwd_workspace_size(C.byref(d)) <= lib.pdb_flash_bwd_noalloc_max_scratch()
        _lib.check(lib.pdb_flash_bwd_noalloc(C.byref(d), stream), "pdb_flash_bwd_noalloc")
        kernels.check_device_errors()
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            err = (a.float() - b.float()).abs().max().item()
            assert err <= BF16_ABS, f"call {call} {name}: {err}"


def test_noalloc_refuses_problems_larger_than_its_scratch(cuda):
    import torch

    from pdum_dsl_b200 import _lib

    lib = _lib.load()
    cap = lib.pdb_flash_bwd_noalloc_max_scratch()
    T = 128
    B = cap // (2 * 4 * T) + 1  # lse2 + D rows alone exceed the scratch
    q = torch.empty(1, 1, T, 64, dtype=torch.bfloat16, device=cuda)
    d = _desc(q, q, q, q, q, None, q, q, q, 0.125, True)
    d.batch = B
    st = lib.pdb_flash_bwd_noalloc(C.byref(d), None)
    assert st == _lib.PDB_ERR_SHAPE
    assert b"fixed scratch" in lib.pdb_last_error_string()
