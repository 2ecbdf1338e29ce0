"""b2_row_reduce_noalloc: the reduction entry point for callers that cannot
allocate device memory (code inside an allocator or out-of-memory handler, or
a runtime that forbids cudaMalloc after start-up). It keeps its scratch in a
fixed array inside the library, so this test calls it through the C ABI with
only caller-owned inputs and outputs and compares it, on two calls in a row,
with b2_row_op given a workspace, and then with the CPU oracle in fp32, fp16
and bf16 over ragged, strided and NaN rows. The file name sorts last so a stop-at-first-
failure run has already run every other test when it gets here."""
import pytest
import torch

from oracle import oracle as O
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


_TDT = {"f32": (torch.float32, _lib.B2_F32), "f16": (torch.float16, _lib.B2_F16),
        "bf16": (torch.bfloat16, _lib.B2_BF16)}


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,cols,pad", [(1, 1000, 0), (7, 65537, 0), (4, 200_000, 24), (2, 1 << 20, 0)])
def test_noalloc_matches_oracle(dt, rows, cols, pad):
    """Against the CPU oracle (float64 sum; max/min values and argmax/argmin
    indices exact), including one split per row (cols < 65536), a ragged last
    chunk, a row pitch wider than the row, a NaN row and lowest-index ties."""
    tdt, code = _TDT[dt]
    L = _lib.lib()
    g = torch.Generator().manual_seed(rows * 7 + cols)
    full = torch.randn(rows, cols + pad, generator=g).to(tdt)
    x_cpu = full[:, :cols]
    if rows > 1:
        x_cpu[1, cols - 1] = 40.0
        x_cpu[1, 3] = 40.0                 # tie: lowest index wins
        x_cpu[1, cols // 2] = -40.0
        x_cpu[1, 5] = -40.0
    if rows > 2:
        x_cpu[2, cols // 3] = float("nan")  # NaN propagates / is the extreme
    xd = full.cuda()
    x = xd[:, :cols]
    for op in ("sum", "max", "min", "argmax", "argmin"):
        idx = op.startswith("arg")
        got = torch.full((rows,), -1, dtype=torch.int64 if idx else tdt, device="cuda")
        for _ in range(2):  # two calls in a row share the scratch array
            st = L.b2_row_reduce_noalloc(_lib.ROW_OPS[op], x.data_ptr(), got.data_ptr(), rows, cols,
                                         x.stride(0), code, _stream())
            _lib.check("b2_row_reduce_noalloc", st)
        torch.cuda.synchronize()
        got = got.cpu()
        if op == "sum":
            # against a float64 sum: fp32 accumulation error relative to sum|x|
            # (as the split-path test of b2_row_op), plus the rounding of the
            # result to the output type (half an ulp: 2^-11 fp16, 2^-8 bf16)
            exact = x_cpu.double().sum(1)
            assert torch.equal(torch.isnan(got.double()), torch.isnan(exact))
            fin = ~torch.isnan(exact)
            store = {"f32": 2.0 ** -24, "f16": 2.0 ** -11, "bf16": 2.0 ** -8}[dt]
            bound = 1e-6 * x_cpu.double().abs().sum(1) + store * exact.abs()
            assert ((got.double() - exact).abs() <= bound)[fin].all(), (got, exact)
        elif op in ("max", "min"):
            ref = getattr(O, f"ref_{op}")(x_cpu).to(tdt)
            assert torch.equal(torch.isnan(got), torch.isnan(ref))
            m = ~torch.isnan(ref)
            assert torch.equal(got[m], ref[m])
        else:
            ref = getattr(O, f"ref_{op}")(x_cpu)
            assert torch.equal(got, ref), (op, got, ref)


def test_noalloc_zero_rows_is_a_no_op():
    L = _lib.lib()
    x = torch.zeros(8, device="cuda")
    assert L.b2_row_reduce_noalloc(_lib.ROW_OPS["sum"], x.data_ptr(), x.data_ptr(), 0, 4, 4,
                                   _lib.B2_F32, _stream()) == _lib.B2_OK


def test_noalloc_rejects_oversize_and_bad_ops():
    L = _lib.lib()
    x = torch.zeros(8, device="cuda")
    # 20000 rows of one chunk each exceeds the 16384-partial scratch
    assert L.b2_row_reduce_noalloc(_lib.ROW_OPS["sum"], x.data_ptr(), x.data_ptr(), 20000, 4, 4,
                                   _lib.B2_F32, _stream()) == _lib.B2_EINVAL
    assert b"exceeds the fixed scratch" in L.b2_last_error()
    assert L.b2_row_reduce_noalloc(_lib.ROW_OPS["softmax"], x.data_ptr(), x.data_ptr(), 1, 4, 4,
                                   _lib.B2_F32, _stream()) == _lib.B2_EINVAL
