"""b2_row_reduce_noalloc: the reduction entry point for callers that cannot
allocate device memory (code inside an allocator or out-of-memory handler, or
a runtime that forbids cudaMalloc after start-up). It keeps its scratch in a
fixed array inside the library, so this test calls it through the C ABI with
only caller-owned inputs and outputs and compares it, on two calls in a row,
with b2_row_op given a workspace. The file name sorts last so a stop-at-first-
failure run has already run every other test when it gets here."""
import pytest
import torch

from triton_msl_b200 import _lib

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _row_op(L, op, x, out):
    rows, cols = x.shape
    code = _lib.ROW_OPS[op]
    ws_bytes = L.b2_query_workspace(1, code, rows, cols, _lib.B2_F32)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    st = L.b2_row_op(code, x.data_ptr(), None, None, out.data_ptr(), rows, cols, x.stride(0), 1,
                     0.0, _lib.B2_F32, ws.data_ptr(), ws_bytes, _stream())
    _lib.check("b2_row_op", st)


@pytest.mark.parametrize("op", ["sum", "max", "min", "argmax", "argmin"])
def test_noalloc_matches_row_op_twice(op):
    L = _lib.lib()
    idx = op.startswith("arg")
    odt = torch.int64 if idx else torch.float32
    for call, (rows, cols) in enumerate([(3, 1 << 20), (5, 300_000)]):
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        x = torch.randn(rows, cols, generator=g, device="cuda")
        x[1, cols // 3] = 50.0       # a clear extreme, tied at a lower index
        x[1, 7] = 50.0
        got = torch.full((rows,), -1, dtype=odt, device="cuda")
        st = L.b2_row_reduce_noalloc(_lib.ROW_OPS[op], x.data_ptr(), got.data_ptr(), rows, cols,
                                     x.stride(0), _lib.B2_F32, _stream())
        _lib.check("b2_row_reduce_noalloc", st)
        ref = torch.empty((rows,), dtype=odt, device="cuda")
        _row_op(L, op, x, ref)
        torch.cuda.synchronize()
        if idx:
            assert torch.equal(got, ref)
        else:
            # fp32 path tolerance of the other GPU tests: max-abs <= 1e-4
            assert (got - ref).abs().max().item() <= 1e-4


def test_noalloc_rejects_oversize_and_bad_ops():
    L = _lib.lib()
    x = torch.zeros(8, device="cuda")
    # 20000 rows of one chunk each exceeds the 16384-partial scratch
    assert L.b2_row_reduce_noalloc(_lib.ROW_OPS["sum"], x.data_ptr(), x.data_ptr(), 20000, 4, 4,
                                   _lib.B2_F32, _stream()) == _lib.B2_EINVAL
    assert b"exceeds the fixed scratch" in L.b2_last_error()
    assert L.b2_row_reduce_noalloc(_lib.ROW_OPS["softmax"], x.data_ptr(), x.data_ptr(), 1, 4, 4,
                                   _lib.B2_F32, _stream()) == _lib.B2_EINVAL
