"""The C-ABI library: builds, loads, exports every declared symbol, validates descriptors (no GPU needed)."""

import ctypes as C
import re
from pathlib import Path

import pytest

from pdum_dsl_b200 import _lib

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "pdb.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(pdb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_exports():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_loads_and_exports_everything():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert _lib.version().startswith("pdb-sm100a")


_STRUCTS = {
    "pdb_rowsoftmax_desc": "RowSoftmaxDesc", "pdb_layernorm_desc": "LayerNormDesc", "pdb_flash_desc": "FlashDesc",
    "pdb_flash_bwd_desc": "FlashBwdDesc", "pdb_ew_op": "EwOp", "pdb_contract_desc": "ContractDesc",
    "pdb_pointwise_desc": "PointwiseDesc", "pdb_sp_op": "SpOp", "pdb_score_program_desc": "ScoreProgramDesc",
}


def test_descriptor_layouts_match_the_header(tmp_path):
    """Every descriptor's size and every field's offset, as a C compiler lays out
    include/pdb.h, equal the ctypes mirror's."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "pdb.h"', "int main(void) {"]
    for cname, pyname in _STRUCTS.items():
        st = getattr(_lib, pyname)
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in st._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                          check=True).stdout.splitlines())
    for cname, pyname in _STRUCTS.items():
        st = getattr(_lib, pyname)
        assert int(got[f"{cname} size"]) == C.sizeof(st), cname
        for fname, _ in st._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(st, fname).offset, f"{cname}.{fname}"


def test_null_descriptors_are_refused():
    lib = _lib.load()
    assert lib.pdb_rowsoftmax_f32(None, None) == _lib.PDB_ERR_ARG
    assert lib.pdb_layernorm_f32(None, None) == _lib.PDB_ERR_ARG
    assert lib.pdb_flash_fwd(None, None) == _lib.PDB_ERR_ARG
    assert b"null descriptor" in lib.pdb_last_error_string()


def test_shape_validation_happens_before_any_launch():
    lib = _lib.load()
    d = _lib.RowSoftmaxDesc(None, None, -1, 4, 4, 4)
    assert lib.pdb_rowsoftmax_f32(C.byref(d), None) == _lib.PDB_ERR_SHAPE
    d = _lib.RowSoftmaxDesc(None, None, 0, 4, 4, 4)  # empty: nothing to do
    assert lib.pdb_rowsoftmax_f32(C.byref(d), None) == _lib.PDB_OK
    f = _lib.FlashDesc()
    f.q = f.k = f.v = f.o = 16
    f.batch, f.heads_q, f.heads_kv, f.seqlen_q, f.seqlen_k, f.head_dim, f.head_dim_v = 1, 3, 2, 8, 8, 64, 64
    assert lib.pdb_flash_fwd(C.byref(f), None) == _lib.PDB_ERR_SHAPE  # 3 q heads over 2 kv heads
    f.heads_q, f.q_start = 4, -1
    assert lib.pdb_flash_fwd(C.byref(f), None) == _lib.PDB_ERR_SHAPE
    f.q_start, f.dtype, f.head_dim, f.head_dim_v = 0, _lib.PDB_BF16, 44, 48  # rows not 16-byte multiples
    assert lib.pdb_flash_fwd(C.byref(f), None) == _lib.PDB_ERR_UNSUPPORTED
    f.head_dim = 264  # above the 256-wide build
    assert lib.pdb_flash_fwd(C.byref(f), None) == _lib.PDB_ERR_UNSUPPORTED
    f.dtype = 7
    assert lib.pdb_flash_fwd(C.byref(f), None) == _lib.PDB_ERR_UNSUPPORTED


def test_python_layer_raises_on_host_tensors():
    import torch

    from pdum_dsl_b200 import kernels

    with pytest.raises(ValueError, match="CUDA"):
        kernels.row_softmax(torch.zeros(2, 2))
    with pytest.raises(ValueError, match="CUDA"):
        kernels.flash_attention(torch.zeros(4, 8), torch.zeros(4, 8), torch.zeros(4, 8))


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.BackendUnavailable):
        _lib.load(tmp_path / "nope.so")


def test_selftest_rejects_unbounded_limits():
    lib = _lib.load()
    assert lib.pdb_selftest_wait_timeout(0, None) == _lib.PDB_ERR_ARG
    assert lib.pdb_selftest_wait_timeout(3_000_000_000, None) == _lib.PDB_ERR_ARG


def _bwd_desc(B, H, HKV, T, D, lse):
    d = _lib.FlashBwdDesc()
    d.q = d.k = d.v = d.o = d.dout = d.dq = d.dk = d.dv = 256
    d.lse = 256 if lse else None
    d.batch, d.heads_q, d.heads_kv, d.seqlen_q, d.seqlen_k, d.head_dim, d.head_dim_v = B, H, HKV, T, T, D, D
    d.scale, d.causal, d.dtype = 0.125, 1, _lib.PDB_BF16
    return d


def test_backward_workspace_sizes():
    """D and nlse2 rows (padded to 128) and two counters; at head_dim 64 also the fused
    pass's fp32 dQ accumulator (64 floats per padded row); without lse the forward's
    recomputed lse and output."""
    lib = _lib.load()
    al = lambda x: (x + 255) // 256 * 256
    B, H, T = 2, 4, 300
    rows = B * H * 384
    base = al(rows * 4) * 2 + al(8)
    assert lib.pdb_flash_bwd_workspace_size(C.byref(_bwd_desc(B, H, 2, T, 128, True))) == base
    assert lib.pdb_flash_bwd_workspace_size(C.byref(_bwd_desc(B, H, 2, T, 64, True))) == base + al(rows * 64 * 4)
    recompute = al(B * H * T * 4) + al(B * H * T * 64 * 2)
    assert lib.pdb_flash_bwd_workspace_size(C.byref(_bwd_desc(B, H, 2, T, 64, False))) == (
        base + al(rows * 64 * 4) + recompute)


def test_backward_refuses_a_small_workspace_before_launching():
    lib = _lib.load()
    d = _bwd_desc(1, 2, 2, 200, 64, True)
    d.workspace, d.workspace_bytes = 256, lib.pdb_flash_bwd_workspace_size(C.byref(d)) - 16
    assert lib.pdb_flash_bwd(C.byref(d), None) == _lib.PDB_ERR_ARG
    assert b"workspace too small" in lib.pdb_last_error_string()


def test_workspace_size_of_a_wrapping_descriptor_is_unsatisfiable():
    """A descriptor whose sizes would overflow the workspace arithmetic reports a
    workspace no caller can provide (SIZE_MAX), so neither entry point launches."""
    lib = _lib.load()
    d = _lib.FlashBwdDesc()
    d.q = d.k = d.v = d.o = d.dout = d.dq = d.dk = d.dv = 16
    d.batch, d.heads_q, d.heads_kv, d.seqlen_q, d.seqlen_k = 1 << 30, 1 << 30, 1 << 30, 1 << 29, 128
    d.head_dim = d.head_dim_v = 64
    d.dtype = _lib.PDB_BF16
    assert lib.pdb_flash_bwd_workspace_size(C.byref(d)) == 2 ** 64 - 1
    assert lib.pdb_flash_bwd_noalloc(C.byref(d), None) != _lib.PDB_OK
