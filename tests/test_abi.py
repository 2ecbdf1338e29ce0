"""C ABI: the library loads, exports exactly what include/b2msl.h declares, and
rejects bad arguments with a status (no GPU needed: validation precedes any
CUDA call)."""
import ctypes
import re
from pathlib import Path

import pytest

from triton_msl_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "b2msl.h"


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert L.b2_version().decode().startswith("b2msl")


def test_row_op_rejects_bad_arguments():
    L = _lib.lib()
    assert L.b2_row_op(99, None, None, None, None, 1, 1, 1, 1, 0.0, 0, None, 0, None) == _lib.B2_EINVAL
    assert b"unknown op" in L.b2_last_error()
    assert L.b2_row_op(0, None, None, None, None, 4, 8, 8, 8, 0.0, 7, None, 0, None) == _lib.B2_EINVAL
    assert L.b2_row_op(0, None, None, None, None, -1, 8, 8, 8, 0.0, 0, None, 0, None) == _lib.B2_EINVAL
    # null pointers with real work
    assert L.b2_row_op(3, None, None, None, None, 4, 8, 8, 8, 0.0, 0, None, 0, None) == _lib.B2_EINVAL
    # row stride smaller than the row
    assert L.b2_row_op(0, 16, None, None, 16, 4, 8, 4, 8, 0.0, 0, None, 0, None) == _lib.B2_EINVAL
    # argmax over empty rows is undefined
    assert L.b2_row_op(5, 16, None, None, 16, 4, 0, 0, 0, 0.0, 0, None, 0, None) == _lib.B2_EINVAL
    # empty work is a successful no-op
    assert L.b2_row_op(0, None, None, None, None, 0, 8, 8, 8, 0.0, 0, None, 0, None) == _lib.B2_OK


def test_gemm_and_fa_reject_bad_arguments():
    L = _lib.lib()
    s6 = _lib.i64_array([1] * 6)
    assert L.b2_gemm(None, None, None, None, -1, 2, 2, s6, 1.0, 0, 0, 0, 0, None, 0, None) == _lib.B2_EINVAL
    assert L.b2_gemm(None, None, None, None, 2, 2, 2, s6, 1.0, 9, 0, 0, 0, None, 0, None) == _lib.B2_EINVAL
    assert L.b2_gemm(None, None, None, None, 2, 2, 2, s6, 1.0, 0, 5, 0, 0, None, 0, None) == _lib.B2_EINVAL
    assert L.b2_gemm(None, None, None, None, 2, 2, 2, s6, 1.0, 0, 0, 0, 0, None, 0, None) == _lib.B2_EINVAL
    assert L.b2_gemm(None, None, None, None, 0, 2, 2, s6, 1.0, 0, 0, 0, 0, None, 0, None) == _lib.B2_OK
    s16 = _lib.i64_array([1] * 16)
    assert L.b2_fa_fwd(None, None, None, None, 1, 1, 8, 0, s16, 1.0, 0, 0, None) == _lib.B2_EINVAL
    assert L.b2_fa_fwd(16, 16, 16, 16, 1, 1, 8, 256, s16, 1.0, 0, 0, None) == _lib.B2_EUNSUPPORTED
    assert L.b2_fa_fwd(16, 16, 16, 16, 1, 1, 8, 64, s16, float("nan"), 0, 0, None) == _lib.B2_EINVAL
    assert L.b2_fa_fwd(None, None, None, None, 1, 1, 0, 64, s16, 1.0, 0, 0, None) == _lib.B2_OK
    with pytest.raises(_lib.B2Unsupported):
        _lib.check("b2_fa_fwd", L.b2_fa_fwd(16, 16, 16, 16, 1, 1, 8, 256, s16, 1.0, 0, 0, None))


def test_workspace_query():
    L = _lib.lib()
    assert L.b2_query_workspace(1, 0, 65536, 4096, 0) == 0       # softmax: none
    assert L.b2_query_workspace(1, 3, 1, 1 << 24, 0) > 0         # 1 x 16M sum: split path
    assert L.b2_query_workspace(0, 8192, 8192, 8192, 1) == 0


def test_fa_host_pipeline_rejects_bad_inputs():
    import torch
    import triton_msl_b200 as b2
    q = torch.zeros(1, 2, 8, 32, dtype=torch.float16)
    with pytest.raises(ValueError):
        b2.flash_attn_fwd_host(q, q, q[:, :1])
    with pytest.raises(ValueError):
        b2.flash_attn_fwd_host(q.transpose(1, 2), q, q)
    with pytest.raises(TypeError):
        b2.flash_attn_fwd_host(q, q.float(), q)
