"""GPU parity of the general fused GEMM epilogue (b2_gemm_epilogue) against the
CPU oracle's restatement of the reference's epilogue op chain
(triton_msl/codegen/_lowerer_templates.py:1733-1855): every op code, on every
GEMM path (CTA pairs, one-SM wide and narrow tiles, split-K, 3xTF32, CUDA
cores), NaN semantics of the propagating and quiet min/max, and exact integer
cases for floor/ceil. Tolerances as the other GPU tests: normwise 2e-3 for
fp16/bf16 inputs (+2^-8 for bf16 outputs), max-abs 1e-4 relative to max|ref|
(floor 1) for fp32."""
import math

import pytest
import torch

import triton_msl_b200 as b2
from oracle import oracle as O
from triton_msl_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(shape, dtype, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype)


def _check(got, ref, in_dtype):
    bf16_out = got.dtype == torch.bfloat16
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref)), "NaN pattern differs"
    m = ~torch.isnan(ref)
    err = (got[m] - ref[m]).abs().max().item()
    scale = max(ref[m].abs().max().item(), 1e-6)
    if in_dtype == torch.float32:
        assert err <= 1e-4 * max(scale, 1.0), f"max-abs {err:.3e}"
    else:
        tol = O.TOL_LOWP_REL + (2.0 ** -8 if bf16_out else 0.0)
        assert err / scale <= tol, f"normwise {err / scale:.3e}"


# ops that need a positive argument get abs + 1 first
_POS = [("abs",), ("add", 1.0)]
CHAINS = {
    "arith": [("add_bias",), ("mul", 0.75), ("add", 0.25), ("sub", 0.1), ("rsub", 2.0), ("div", 3.0)],
    "rdiv": _POS + [("rdiv", 1.5)],
    "bias_mul": [("mul_bias",), ("fma", 2.0, -0.5)],
    "minmax": [("max", -0.2), ("min", 0.3), ("maxnum", -0.1), ("minnum", 0.2)],
    "clamp": [("clamp", -0.5, 0.5), ("clampnum", -0.25, 0.4)],
    "exp_log": [("neg",), ("exp",), ("log",), ("exp2",)] + _POS + [("log2",)],
    "roots": _POS + [("sqrt",), ("rsqrt",)],
    "trig": [("mul", 3.0), ("sin",), ("cos",)],
    "acts": [("erf",), ("tanh",), ("relu",), ("gelu",), ("gelu_tanh",), ("silu",), ("sigmoid",)],
    "abs": [("abs",), ("neg",)],
}


@pytest.mark.parametrize("chain", sorted(CHAINS))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_epilogue_ops_match_oracle(chain, dtype):
    M, N, K = 384, 640, 512
    a = _rand((M, K), dtype, 1, 1 / math.sqrt(K))
    b = _rand((K, N), dtype, 2, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 3, 0.5)
    ops = CHAINS[chain]
    c = b2.gemm_epilogue(a.to(DEV), b.to(DEV), ops, bias.to(DEV), torch.float32)
    _check(c, O.ref_gemm_epilogue(a, b, ops, bias, torch.float32), dtype)


# each GEMM path, with one chain that touches bias, constants and a transcendental
_PATH_OPS = [("add_bias",), ("mul", 1.5), ("gelu",), ("clamp", -0.3, 2.0), ("fma", 0.5, 0.1)]


@pytest.mark.parametrize("M,N,K,dtype,out_dtype,variant", [
    (2304, 2304, 1024, torch.bfloat16, torch.bfloat16, "gemm_sm100_pair"),
    (2048, 2048, 512, torch.float16, torch.float16, "gemm_sm100"),
    (512, 4096, 1024, torch.float16, torch.float32, "gemm_sm100_n128"),
    (256, 256, 8192, torch.bfloat16, torch.float32, "gemm_sm100_splitk"),
    (300, 200, 264, torch.float32, torch.float32, "gemm_sm100_tf32x3"),
    (1024, 512, 1024, torch.float32, torch.float32, "gemm_sm100_tf32x3"),
])
def test_epilogue_on_every_gemm_path(M, N, K, dtype, out_dtype, variant):
    a = _rand((M, K), dtype, 11, 1 / math.sqrt(K))
    b = _rand((K, N), dtype, 12, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 13, 0.5)
    c = b2.gemm_epilogue(a.to(DEV), b.to(DEV), _PATH_OPS, bias.to(DEV), out_dtype)
    assert b2.last_kernel() == variant
    _check(c, O.ref_gemm_epilogue(a, b, _PATH_OPS, bias, out_dtype), dtype)


def test_epilogue_cuda_core_path_and_k_major_b():
    a = _rand((200, 130), torch.float16, 21, 0.1)[:, :129]  # odd row pitch: CUDA cores
    w = _rand((96, 129), torch.float16, 22, 0.1)
    bias = _rand((96,), torch.float16, 23, 0.5)
    ops = [("add_bias",), ("silu",), ("max", 0.01)]
    c = b2.gemm_epilogue(a.to(DEV), w.to(DEV).t(), ops, bias.to(DEV))
    assert b2.last_kernel() == "gemm_simt"
    _check(c, O.ref_gemm_epilogue(a, w.t(), ops, bias, torch.float16), torch.float16)


def test_epilogue_nan_propagating_and_quiet():
    M, N, K = 256, 384, 256
    a = _rand((M, K), torch.float16, 31, 1 / 16)
    a[5, 7] = float("nan")               # row 5 of the product is NaN
    b = _rand((K, N), torch.float16, 32, 1 / 16)
    for ops in ([("max", 0.0)], [("maxnum", 0.0)], [("min", 0.0)], [("minnum", 0.0)],
                [("clamp", -0.1, 0.1)], [("clampnum", -0.1, 0.1)], [("relu",)]):
        c = b2.gemm_epilogue(a.to(DEV), b.to(DEV), ops, None, torch.float32)
        ref = O.ref_gemm_epilogue(a, b, ops, None, torch.float32)
        _check(c, ref, torch.float16)
        quiet = ops[0][0] in ("maxnum", "minnum", "clampnum")
        assert bool(torch.isnan(c[5]).all()) != quiet


def test_epilogue_floor_ceil_exact_on_integer_products():
    # small integers: the products and sums are exact, so floor/ceil compare exactly
    g = torch.Generator().manual_seed(41)
    a = torch.randint(-3, 4, (256, 128), generator=g).half()
    b = torch.randint(-3, 4, (128, 384), generator=g).half()
    for ops in ([("mul", 0.37), ("floor",)], [("mul", 0.37), ("ceil",)], [("div", 3.0), ("floor",), ("abs",)]):
        c = b2.gemm_epilogue(a.to(DEV), b.to(DEV), ops, None, torch.float32)
        assert torch.equal(c.cpu(), O.ref_gemm_epilogue(a, b, ops, None, torch.float32))


def test_epilogue_rejects_bad_programs():
    x = torch.zeros(128, 128, device=DEV, dtype=torch.float16)
    with pytest.raises(ValueError):
        b2.gemm_epilogue(x, x, [("nope",)])
    with pytest.raises(ValueError):
        b2.gemm_epilogue(x, x, [("add",)])          # missing constant
    with pytest.raises(ValueError):
        b2.gemm_epilogue(x, x, [("neg",)] * 17)     # too many ops
    with pytest.raises(_lib.B2Error):
        b2.gemm_epilogue(x, x, [("add_bias",)])     # no bias given
    assert b2.device_status(0) == 0
