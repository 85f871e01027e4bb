"""ctypes binding of the C ABI declared in ``include/pdb.h``.

The library is the in-tree ``libpdb_sm100.so`` built by ``pdum_dsl_b200.build``.
There is no fallback: if the library is missing or fails to load, every
entry point raises ``BackendUnavailable``.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpdb_sm100.so"

PDB_OK, PDB_ERR_SHAPE, PDB_ERR_ALIGN, PDB_ERR_TIMEOUT, PDB_ERR_CUDA, PDB_ERR_UNSUPPORTED, PDB_ERR_ARG = range(7)
PDB_F32, PDB_BF16 = 0, 1

STATUS_NAMES = {
    PDB_OK: "PDB_OK",
    PDB_ERR_SHAPE: "PDB_ERR_SHAPE",
    PDB_ERR_ALIGN: "PDB_ERR_ALIGN",
    PDB_ERR_TIMEOUT: "PDB_ERR_TIMEOUT",
    PDB_ERR_CUDA: "PDB_ERR_CUDA",
    PDB_ERR_UNSUPPORTED: "PDB_ERR_UNSUPPORTED",
    PDB_ERR_ARG: "PDB_ERR_ARG",
}

# every symbol include/pdb.h declares
EXPORTS = (
    "pdb_rowsoftmax_f32",
    "pdb_layernorm_f32",
    "pdb_flash_fwd",
    "pdb_flash_bwd",
    "pdb_flash_bwd_workspace_size",
    "pdb_flash_bwd_noalloc",
    "pdb_flash_bwd_noalloc_max_scratch",
    "pdb_contract",
    "pdb_pointwise_f32",
    "pdb_score_program_f32",
    "pdb_check_error",
    "pdb_selftest_wait_timeout",
    "pdb_last_error_string",
    "pdb_version",
)


class BackendUnavailable(RuntimeError):
    """The sm_100a kernel library is not built / not loadable."""


class PdbError(RuntimeError):
    """A non-OK status from the C ABI."""

    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}: {detail}")
        self.status = status


I64x3 = C.c_int64 * 3


class RowSoftmaxDesc(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("y", C.c_void_p),
        ("rows", C.c_int64),
        ("cols", C.c_int64),
        ("x_row_stride", C.c_int64),
        ("y_row_stride", C.c_int64),
    ]


class LayerNormDesc(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("gamma", C.c_void_p),
        ("beta", C.c_void_p),
        ("y", C.c_void_p),
        ("rows", C.c_int64),
        ("cols", C.c_int64),
        ("x_row_stride", C.c_int64),
        ("y_row_stride", C.c_int64),
        ("eps", C.c_double),
    ]


class FlashDesc(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
        ("o", C.c_void_p),
        ("lse", C.c_void_p),
        ("m", C.c_void_p),
        ("den", C.c_void_p),
        ("batch", C.c_int64),
        ("heads_q", C.c_int64),
        ("heads_kv", C.c_int64),
        ("seqlen_q", C.c_int64),
        ("seqlen_k", C.c_int64),
        ("head_dim", C.c_int64),
        ("head_dim_v", C.c_int64),
        ("q_stride", I64x3),
        ("k_stride", I64x3),
        ("v_stride", I64x3),
        ("o_stride", I64x3),
        ("q_start", C.c_int64),
        ("scale", C.c_double),
        ("causal", C.c_int32),
        ("dtype", C.c_int32),
        ("key_lo", C.c_void_p),
        ("key_hi", C.c_void_p),
        ("mask_monotone", C.c_int32),
        ("sm_margin", C.c_int32),
    ]


class FlashBwdDesc(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
        ("o", C.c_void_p),
        ("dout", C.c_void_p),
        ("lse", C.c_void_p),
        ("dq", C.c_void_p),
        ("dk", C.c_void_p),
        ("dv", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("batch", C.c_int64),
        ("heads_q", C.c_int64),
        ("heads_kv", C.c_int64),
        ("seqlen_q", C.c_int64),
        ("seqlen_k", C.c_int64),
        ("head_dim", C.c_int64),
        ("head_dim_v", C.c_int64),
        ("q_stride", I64x3),
        ("k_stride", I64x3),
        ("v_stride", I64x3),
        ("o_stride", I64x3),
        ("do_stride", I64x3),
        ("dq_stride", I64x3),
        ("dk_stride", I64x3),
        ("dv_stride", I64x3),
        ("q_start", C.c_int64),
        ("scale", C.c_double),
        ("causal", C.c_int32),
        ("dtype", C.c_int32),
    ]


EW_OPS = {"add": 1, "sub": 2, "mul": 3, "div": 4, "maximum": 5, "minimum": 6, "exp": 7, "log": 8, "sqrt": 9,
          "tanh": 10, "neg": 11}
MAX_EW_OPS = 8


class EwOp(C.Structure):
    _fields_ = [
        ("op", C.c_int32),
        ("operand", C.c_int32),
        ("swap", C.c_int32),
        ("reserved", C.c_int32),
        ("value", C.c_double),
        ("ptr", C.c_void_p),
        ("stride", I64x3),
    ]


class ContractDesc(C.Structure):
    _fields_ = [
        ("a", C.c_void_p),
        ("b", C.c_void_p),
        ("c", C.c_void_p),
        ("batch", C.c_int64),
        ("m", C.c_int64),
        ("n", C.c_int64),
        ("k", C.c_int64),
        ("a_stride", I64x3),
        ("b_stride", I64x3),
        ("c_stride", I64x3),
        ("alpha", C.c_double),
        ("dtype", C.c_int32),
        ("n_ops", C.c_int32),
        ("ops", EwOp * MAX_EW_OPS),
    ]


class PointwiseDesc(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("y", C.c_void_p),
        ("batch", C.c_int64),
        ("m", C.c_int64),
        ("n", C.c_int64),
        ("x_stride", I64x3),
        ("y_stride", I64x3),
        ("n_ops", C.c_int32),
        ("reserved", C.c_int32),
        ("ops", EwOp * MAX_EW_OPS),
    ]


# score-space programs (pdb_score_program_f32)
SP_OPS = {"score": 1, "row": 2, "col": 3, "tile": 4, "iota_row": 5, "iota_col": 6, "const": 7, "where": 8,
          "add": 9, "sub": 10, "mul": 11, "div": 12, "maximum": 13, "minimum": 14, "le": 15, "lt": 16, "ge": 17,
          "gt": 18, "eq": 19, "ne": 20, "and": 21, "or": 22,
          "exp": 23, "log": 24, "neg": 25, "recip": 26, "sqrt": 27, "tanh": 28, "not": 29, "abs": 30,
          "floor": 31}
SP_UNARY = ("exp", "log", "neg", "recip", "sqrt", "tanh", "not", "abs", "floor")
SP_OUT = {"tile": 0, "row_sum": 1, "row_max": 2, "row_min": 3, "row_contract": 4}
SP_MAX_OPS, SP_MAX_REGS, SP_MAX_SCORES, SP_MAX_VECS, SP_MAX_TILES = 64, 12, 2, 6, 4
I64x4 = C.c_int64 * 4
I64x5 = C.c_int64 * 5


class SpOp(C.Structure):
    _fields_ = [
        ("op", C.c_int32),
        ("dst", C.c_int32),
        ("a", C.c_int32),
        ("b", C.c_int32),
        ("c", C.c_int32),
        ("reserved", C.c_int32),
        ("value", C.c_double),
    ]


class ScoreProgramDesc(C.Structure):
    _fields_ = [
        ("batch", C.c_int64),
        ("batch_mid", C.c_int64),
        ("batch_inner", C.c_int64),
        ("rows", C.c_int64),
        ("cols", C.c_int64),
        ("row_start", C.c_int64),
        ("col_start", C.c_int64),
        ("n_scores", C.c_int32),
        ("n_ops", C.c_int32),
        ("n_regs", C.c_int32),
        ("result", C.c_int32),
        ("score_a", C.c_void_p * SP_MAX_SCORES),
        ("score_b", C.c_void_p * SP_MAX_SCORES),
        ("score_feat", C.c_int64 * SP_MAX_SCORES),
        ("score_a_stride", I64x5 * SP_MAX_SCORES),
        ("score_b_stride", I64x5 * SP_MAX_SCORES),
        ("rowvec", C.c_void_p * SP_MAX_VECS),
        ("rowvec_stride", I64x4 * SP_MAX_VECS),
        ("colvec", C.c_void_p * SP_MAX_VECS),
        ("colvec_stride", I64x4 * SP_MAX_VECS),
        ("tile", C.c_void_p * SP_MAX_TILES),
        ("tile_stride", I64x5 * SP_MAX_TILES),
        ("ops", SpOp * SP_MAX_OPS),
        ("out_mode", C.c_int32),
        ("reserved", C.c_int32),
        ("out", C.c_void_p),
        ("out_stride", I64x5),
        ("w", C.c_void_p),
        ("w_stride", I64x5),
        ("xdim", C.c_int64),
    ]


_LIB = None


def load(path: Path | None = None) -> C.CDLL:
    """Load (once) and type the library; raise BackendUnavailable if absent."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise BackendUnavailable(
            f"{p.name} is not built: run `python -m pdum_dsl_b200.build` (nvcc, sm_100a); "
            "there is no CPU or library fallback"
        )
    try:
        lib = C.CDLL(str(p))
    except OSError as e:  # pragma: no cover - depends on the host
        raise BackendUnavailable(f"cannot load {p}: {e}") from e
    vp = C.c_void_p
    lib.pdb_rowsoftmax_f32.argtypes = [C.POINTER(RowSoftmaxDesc), vp]
    lib.pdb_layernorm_f32.argtypes = [C.POINTER(LayerNormDesc), vp]
    lib.pdb_flash_fwd.argtypes = [C.POINTER(FlashDesc), vp]
    lib.pdb_flash_bwd.argtypes = [C.POINTER(FlashBwdDesc), vp]
    lib.pdb_flash_bwd_workspace_size.argtypes = [C.POINTER(FlashBwdDesc)]
    lib.pdb_flash_bwd_workspace_size.restype = C.c_size_t
    lib.pdb_flash_bwd_noalloc.argtypes = [C.POINTER(FlashBwdDesc), vp]
    lib.pdb_flash_bwd_noalloc_max_scratch.argtypes = []
    lib.pdb_flash_bwd_noalloc_max_scratch.restype = C.c_size_t
    lib.pdb_contract.argtypes = [C.POINTER(ContractDesc), vp]
    lib.pdb_pointwise_f32.argtypes = [C.POINTER(PointwiseDesc), vp]
    lib.pdb_score_program_f32.argtypes = [C.POINTER(ScoreProgramDesc), vp]
    lib.pdb_check_error.argtypes = [vp]
    lib.pdb_selftest_wait_timeout.argtypes = [C.c_int64, vp]
    lib.pdb_last_error_string.restype = C.c_char_p
    lib.pdb_version.restype = C.c_char_p
    for name in EXPORTS:
        f = getattr(lib, name)
        if name not in ("pdb_flash_bwd_workspace_size", "pdb_flash_bwd_noalloc_max_scratch",
                        "pdb_last_error_string", "pdb_version"):
            f.restype = C.c_int
    if path is None:
        _LIB = lib
    return lib


def check(status: int, what: str) -> None:
    if status != PDB_OK:
        detail = load().pdb_last_error_string().decode(errors="replace")
        raise PdbError(status, what, detail)


def version() -> str:
    return load().pdb_version().decode()
