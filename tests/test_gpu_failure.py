"""Failure detection without a GPU fault: a bounded device wait that runs out
reports PDB_ERR_TIMEOUT through the error word, and the context stays usable."""

import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_survives(cuda):
    import torch

    from pdum_dsl_b200 import _lib, kernels

    lib = _lib.load()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.pdb_check_error(s) == _lib.PDB_OK
    assert lib.pdb_selftest_wait_timeout(50_000_000, s) == _lib.PDB_OK  # 50 ms
    assert lib.pdb_check_error(s) == _lib.PDB_ERR_TIMEOUT
    assert b"bounded device wait expired" in lib.pdb_last_error_string()
    assert lib.pdb_check_error(s) == _lib.PDB_OK  # the flag was cleared
    x = torch.randn(4, 256, device=cuda)
    y = kernels.row_softmax(x)  # the context still works
    assert torch.allclose(y.sum(1), torch.ones(4, device=cuda), atol=1e-5)
