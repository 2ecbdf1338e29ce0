"""GPU tests of two host-visible contracts of the C ABI:

* bounded device waits: a tensor-core GEMM whose loader is told to load
  nothing must give up after its (short) wait limit, report B2_ETIMEOUT with
  the TMA bit through b2_device_status, leave the context usable, and a normal
  call afterwards must still match the oracle. This is the device side of the
  reference's "fast path fails -> report, do not hang" contract
  (triton_msl/autotuning/_fast_matmul_dispatch.py:152-158); the failure is made
  by a flag nothing sets, never by a fault.
* re-entrancy: FA, GEMM and row ops called from four host threads, each on its
  own CUDA stream, give the same results as the oracle.
"""
import ctypes
import threading

import pytest
import torch

import triton_msl_b200 as b2
from oracle import oracle as O
from triton_msl_b200 import _lib

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype)


@pytest.mark.parametrize("shape", [(128, 256, 64), (512, 512, 1024)])
def test_bounded_wait_expires_and_reports(shape):
    M, N, K = shape
    L = _lib.lib()
    dev = torch.cuda.current_device()
    _lib.device_status(dev, clear=True)
    a = torch.randn(M, K, device="cuda").half()
    bt = torch.randn(N, K, device="cuda").half()
    c = torch.zeros(M, N, device="cuda", dtype=torch.float16)
    st = L.b2_test_stalled_gemm(a.data_ptr(), bt.data_ptr(), c.data_ptr(), M, N, K,
                                50_000, torch.cuda.current_stream().cuda_stream)
    _lib.check("b2_test_stalled_gemm", st)
    out = ctypes.c_uint32(0)
    rc = L.b2_device_status(dev, 0, ctypes.byref(out))
    assert rc == _lib.B2_ETIMEOUT
    bits = int(out.value)
    assert bits & _lib.STATUS_TIMEOUT_TMA, f"status bits {bits:#x}"
    # nothing was computed: C keeps its zeros
    assert torch.count_nonzero(c).item() == 0
    # clear resets the word
    assert _lib.device_status(dev, clear=True) & _lib.STATUS_TIMEOUT_TMA
    assert _lib.device_status(dev, clear=False) == 0
    # the context is still usable and a normal call matches the oracle
    ref = O.ref_gemm(a.cpu(), bt.cpu().t(), None, "none", torch.float16)
    got = b2.gemm(a, bt.t(), None, "none", torch.float16)
    assert b2.last_kernel().startswith("gemm_sm100")
    assert O.normwise_err(got, ref) <= O.TOL_LOWP_REL
    assert _lib.device_status(dev, clear=True) == 0


def test_stalled_gemm_rejects_bad_arguments():
    L = _lib.lib()
    a = torch.zeros(128, 64, device="cuda", dtype=torch.float16)
    assert L.b2_test_stalled_gemm(a.data_ptr(), a.data_ptr(), a.data_ptr(), 128, 128, 64, 0,
                                  None) == _lib.B2_EINVAL
    assert L.b2_test_stalled_gemm(a.data_ptr(), a.data_ptr(), a.data_ptr(), 128, 128, 63, 1000,
                                  None) == _lib.B2_EINVAL
    assert L.b2_test_stalled_gemm(a.data_ptr(), a.data_ptr(), a.data_ptr(), 128, 128, 64,
                                  2_000_000_000, None) == _lib.B2_EINVAL


def test_ops_from_four_host_threads_on_four_streams():
    cases = []
    for t in range(4):
        q, k, v = (_rand((1, 4, 384, 128), torch.float16, 10 * t + s, 0.5) for s in range(3))
        a = _rand((640, 512), torch.bfloat16, 50 + t, 0.05)
        bm = _rand((512, 768), torch.bfloat16, 60 + t, 0.05)
        bias = _rand((768,), torch.float32, 70 + t, 0.1)
        x = _rand((300, 4096 + 8 * t), torch.float32, 80 + t)
        refs = (O.ref_attention(q, k, v, True), O.ref_gemm(a, bm, bias, "relu", torch.bfloat16),
                O.ref_softmax(x), O.ref_argmax(x), O.ref_rmsnorm(x, None, 1e-6))
        cases.append(((q.cuda(), k.cuda(), v.cuda()), (a.cuda(), bm.cuda(), bias.cuda()),
                      x.cuda(), refs))
    results = [None] * 4
    errors = []
    barrier = threading.Barrier(4)

    def work(t):
        try:
            s = torch.cuda.Stream()
            (q, k, v), (a, bm, bias), x, _ = cases[t]
            barrier.wait()
            with torch.cuda.stream(s):
                outs = []
                for _ in range(5):  # repeat so the threads' launches interleave
                    outs = [b2.flash_attn_fwd(q, k, v, causal=True),
                            b2.gemm(a, bm, bias, "relu", torch.bfloat16),
                            b2.row_softmax(x), b2.row_argmax(x), b2.row_rmsnorm(x, None, 1e-6)]
            s.synchronize()
            results[t] = [o.cpu() for o in outs]
        except Exception as e:  # surfaced below
            errors.append((t, repr(e)))

    threads = [threading.Thread(target=work, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not errors, errors
    for t in range(4):
        got = results[t]
        ref = cases[t][3]
        assert O.normwise_err(got[0], ref[0]) <= O.TOL_LOWP_REL
        assert O.normwise_err(got[1], ref[1]) <= O.TOL_LOWP_REL + 2.0 ** -8
        assert O.max_abs_err(got[2], ref[2]) <= O.TOL_F32_ABS
        assert torch.equal(got[3], ref[3])
        assert O.max_abs_err(got[4], ref[4]) <= O.TOL_F32_ABS
    assert _lib.device_status(torch.cuda.current_device(), clear=True) == 0
