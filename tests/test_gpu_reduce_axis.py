"""GPU parity of reductions along a non-last axis (b2_reduce_axis) against the
CPU oracle (the reference fuzzer's forms A.float().sum(0) and friends,
tests/test_fuzz_reduce.py:88-139): 2-D and 3-D inputs along axes 0 and 1, fp32 /
fp16 / bf16, the split path (long axis, small output) with and without its
workspace, NaN and tie rules, and empty axes. Tolerances as the other GPU tests:
sums against a float64 sum relative to sum|x| (1e-6) plus the output rounding;
max/min values and argmax/argmin indices exact."""
import pytest
import torch

import triton_msl_b200 as b2
from oracle import oracle as O
from triton_msl_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
STORE = {torch.float32: 2.0 ** -24, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


def _rand(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _check(got, x, op, dim):
    got = got.cpu()
    if op == "sum":
        exact = x.double().sum(dim)
        assert torch.equal(torch.isnan(got.double()), torch.isnan(exact))
        fin = ~torch.isnan(exact)
        bound = 1e-6 * x.double().abs().sum(dim) + STORE[x.dtype] * exact.abs() + 1e-30
        assert ((got.double() - exact).abs() <= bound)[fin].all()
    elif op in ("max", "min"):
        ref = O.ref_reduce_axis(x, op, dim).to(x.dtype)
        assert torch.equal(torch.isnan(got), torch.isnan(ref))
        assert torch.equal(got[~torch.isnan(ref)], ref[~torch.isnan(ref)])
    else:
        assert torch.equal(got, O.ref_reduce_axis(x, op, dim))


@pytest.mark.parametrize("op", ["sum", "max", "min", "argmax", "argmin"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape,dim", [((512, 1000), 0), ((4096, 12), 0), ((6, 700, 33), 1),
                                       ((3000, 5, 64), 0), ((64, 8, 4096), 1), ((2, 65536, 8), 1)])
def test_reduce_axis_matches_oracle(op, dtype, shape, dim):
    x = _rand(shape, dtype, sum(shape) + dim)
    got = b2.reduce(x.to(DEV), op, dim)
    assert b2.last_kernel() == "axis_reduce"
    _check(got, x, op, dim)


def test_reduce_axis_nan_ties_and_split_without_workspace():
    x = torch.randn(8192, 24)
    x[100, 3] = x[7000, 3] = 50.0          # tie: lower index
    x[17, 5] = float("nan")                # NaN is the extreme, propagates
    x[4000, 9] = -60.0
    x[9, 9] = -60.0
    xd = x.to(DEV)
    for op in ("sum", "max", "min", "argmax", "argmin"):
        got = b2.reduce(xd, op, 0)
        _check(got, x, op, 0)
    L = _lib.lib()
    assert L.b2_query_workspace(3, 1, 8192, 24, 0) > 0       # this shape splits the axis
    out = torch.empty(24, dtype=torch.int64, device=DEV)
    st = L.b2_reduce_axis(_lib.ROW_OPS["argmax"], xd.data_ptr(), out.data_ptr(), 1, 8192, 24,
                          _lib.B2_F32, None, 0, torch.cuda.current_stream().cuda_stream)
    _lib.check("b2_reduce_axis", st)
    assert torch.equal(out.cpu(), O.ref_reduce_axis(x, "argmax", 0))


def test_reduce_axis_edge_shapes():
    assert b2.reduce(torch.zeros(0, 5, device=DEV), "sum", 0).tolist() == [0.0] * 5
    assert b2.reduce(torch.ones(4, 0, 3, device=DEV), "sum", 1).tolist() == [[0.0] * 3] * 4
    with pytest.raises(b2.B2Error):
        b2.reduce(torch.ones(4, 0, 3, device=DEV), "max", 1)
    assert b2.reduce(torch.ones(3, 1, device=DEV), "argmax", 0).tolist() == [0]
    assert b2.device_status(0) == 0
