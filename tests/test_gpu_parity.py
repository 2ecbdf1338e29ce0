"""GPU parity: every kernel family against the CPU oracle on the same seeded inputs.

Tolerances (written per test): fp32 paths max-abs <= 1e-4; fp16/bf16 paths
normwise-relative <= 2e-3 (max|got-ref| / max|ref|); argmax/argmin bit-exact.
Cases mirror the reference's parity tests: FA over dtype x causal x unaligned N
(tests/test_fa_simdgroup_diff.py:38-57), matmul shapes of
tests/test_fast_matmul_parity.py:47-62, reduce forms of tests/test_fuzz_reduce.py.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import triton_msl_b200 as b2
from oracle import oracle as O
from triton_msl_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
F32_ABS, LOWP_REL = O.TOL_F32_ABS, O.TOL_LOWP_REL
# A bf16 result rounded from the exact value is already up to 2^-8 (half an
# ulp) away from it, relative to its own magnitude, so bf16 outputs get that
# storage allowance on top of the 2e-3 arithmetic bound.
BF16_STORE = 2.0 ** -8


def _rand(shape, dtype, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype)


def _check(got, ref, dtype):
    if dtype == torch.float32 and got.dtype == torch.float32:
        err = O.max_abs_err(got, ref)
        assert err <= F32_ABS, f"max-abs {err:.3e} > {F32_ABS}"
    else:
        tol = LOWP_REL + (BF16_STORE if got.dtype == torch.bfloat16 else 0.0)
        err = O.normwise_err(got, ref)
        assert err <= tol, f"normwise {err:.3e} > {tol:.3e}"


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [50, 100, 128, 192, 256, 600])
def test_fa_tensor_core_matches_oracle(dtype, D, causal, S):
    q, k, v = (_rand((1, 2, S, D), dtype, s, 0.5) for s in (1, 2, 3))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    assert b2.last_kernel() == "fa_sm100"
    _check(o, O.ref_attention(q, k, v, causal), dtype)


@pytest.mark.parametrize("D", [64, 128])
def test_fa_long_sequence_bf16_causal(D):
    q, k, v = (_rand((2, 2, 2048, D), torch.bfloat16, s, 0.5) for s in (4, 5, 6))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=True)
    assert b2.last_kernel() == "fa_sm100"
    _check(o, O.ref_attention(q, k, v, True), torch.bfloat16)


def test_fa_config1_fp32():
    """benchmark configuration 1: fp32 non-causal [1,4,256,64], N(0,1) seed 0, scale 1/8."""
    q, k, v = W.fa_inputs(W.FA_F32, seed=0)
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=False, sm_scale=1 / 8)
    assert b2.last_kernel() == "fa_simt"
    _check(o, O.ref_attention(q, k, v, False, 1 / 8), torch.float32)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S,D", [(50, 32), (100, 64), (192, 128), (77, 48)])
def test_fa_fp32_unaligned(causal, S, D):
    q, k, v = (_rand((2, 3, S, D), torch.float32, s) for s in (7, 8, 9))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    _check(o, O.ref_attention(q, k, v, causal), torch.float32)


def test_fa_strided_layouts():
    """[B,S,H,D] storage viewed as [B,H,S,D] stays on tensor cores; a non-unit
    inner stride goes to the CUDA-core kernel. Both must match."""
    base = _rand((2, 300, 4, 128), torch.float16, 11, 0.5).to(DEV)
    q = base.permute(0, 2, 1, 3)
    k = _rand((2, 300, 4, 128), torch.float16, 12, 0.5).to(DEV).permute(0, 2, 1, 3)
    v = _rand((2, 300, 4, 128), torch.float16, 13, 0.5).to(DEV).permute(0, 2, 1, 3)
    o = b2.flash_attn_fwd(q, k, v, causal=True)
    assert b2.last_kernel() == "fa_sm100"
    ref = O.ref_attention(q.cpu(), k.cpu(), v.cpu(), True)
    _check(o, ref, torch.float16)
    qs = _rand((1, 2, 64, 128 * 2), torch.float16, 14, 0.5).to(DEV)[..., ::2]
    ks = _rand((1, 2, 64, 128), torch.float16, 15, 0.5).to(DEV)
    vs = _rand((1, 2, 64, 128), torch.float16, 16, 0.5).to(DEV)
    o2 = b2.flash_attn_fwd(qs, ks, vs, causal=False)
    assert b2.last_kernel() == "fa_simt"
    _check(o2, O.ref_attention(qs.cpu(), ks.cpu(), vs.cpu(), False), torch.float16)


def test_fa_custom_scale():
    q, k, v = (_rand((1, 2, 256, 64), torch.float16, s, 0.5) for s in (21, 22, 23))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=True, sm_scale=0.3)
    _check(o, O.ref_attention(q, k, v, True, 0.3), torch.float16)


def test_fa_golden_fixtures():
    gold = np.load(Path(__file__).parent / "golden" / "golden.npz")
    meta = json.loads(bytes(gold["__meta__"]).decode())
    for m in meta:
        if not m["name"].startswith("fa_"):
            continue
        t = {k: torch.from_numpy(gold[f"{m['name']}/{k}"].copy()) for k in "qkvo"}
        causal = bool(gold[f"{m['name']}/causal"])
        o = b2.flash_attn_fwd(t["q"].to(DEV), t["k"].to(DEV), t["v"].to(DEV), causal=causal)
        _check(o, t["o"], t["q"].dtype)


# ----------------------------------------------------------------------- gemm
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (512, 512, 512), (256, 2080, 256),
                                   (256, 256, 264), (1024, 512, 256), (300, 200, 136)])
def test_gemm_tensor_core_matches_oracle(dtype, M, N, K):
    a = _rand((M, K), dtype, 31, 1 / math.sqrt(K))
    b = _rand((K, N), dtype, 32, 1 / math.sqrt(K))
    c = b2.gemm(a.to(DEV), b.to(DEV))
    assert b2.last_kernel().startswith("gemm_sm100")
    _check(c, O.ref_gemm(a, b, out_dtype=torch.float32), dtype)


@pytest.mark.parametrize("act", ["none", "relu", "gelu", "gelu_tanh", "silu"])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16])
def test_gemm_epilogue(act, out_dtype):
    M, N, K = 384, 640, 512
    a = _rand((M, K), torch.float16, 41, 1 / math.sqrt(K))
    b = _rand((K, N), torch.float16, 42, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 43, 0.1)
    c = b2.gemm(a.to(DEV), b.to(DEV), bias.to(DEV), act, out_dtype)
    assert c.dtype == out_dtype
    _check(c, O.ref_gemm(a, b, bias, act, torch.float32), torch.float16)


# Occupancy-aware tile choice (reference matmul_tuner.py:76-104): few output
# tiles with a long K split the K loop across CTAs; shapes whose last wave of
# 128x256 tiles would idle more SMs take 128x128 tiles.
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K,b_kmajor,variant", [
    (256, 256, 8192, False, "gemm_sm100_splitk"),
    (100, 296, 5008, False, "gemm_sm100_splitk"),   # ragged M, N; uneven K ranges
    (64, 1001, 2048, True, "gemm_sm100_splitk"),    # N not a multiple of 4 (K-major B)
    (1024, 1024, 4096, False, "gemm_sm100_splitk"),
    (512, 4096, 4096, False, "gemm_sm100_n128"),    # < 1 wave of 128x256 tiles
    (1000, 1500, 320, True, "gemm_sm100_n128"),
    (512, 512, 256, False, "gemm_sm100_n128"),      # K too short to split
    (4096, 4096, 512, False, "gemm_sm100_pair"),
])
def test_gemm_tile_choice_paths(dtype, M, N, K, b_kmajor, variant):
    a = _rand((M, K), dtype, 61, 1 / math.sqrt(K))
    if b_kmajor:
        w = _rand((N, K), dtype, 62, 1 / math.sqrt(K))
        b = w.t()
        c = b2.gemm(a.to(DEV), w.to(DEV).t())
    else:
        b = _rand((K, N), dtype, 62, 1 / math.sqrt(K))
        c = b2.gemm(a.to(DEV), b.to(DEV))
    assert b2.last_kernel() == variant
    _check(c, O.ref_gemm(a, b, out_dtype=torch.float32), dtype)


# Shapes with a full wave of 256x256 tiles run on CTA pairs (tcgen05
# cta_group::2, M=256 MMAs): ragged M/N/K, both B layouts, epilogues, outputs.
@pytest.mark.parametrize("M,N,K,b_kmajor,act,out_dtype,dtype", [
    (2000, 2504, 1000, False, "relu", torch.float16, torch.float16),
    (2000, 2504, 1000, True, "gelu", torch.bfloat16, torch.bfloat16),
    (2304, 2304, 2048, False, "none", torch.float32, torch.bfloat16),
    (2304, 2304, 2048, True, "silu", torch.float32, torch.float16),
    (4100, 2056, 520, True, "gelu_tanh", torch.float16, torch.float16),
])
def test_gemm_pair_paths(M, N, K, b_kmajor, act, out_dtype, dtype):
    a = _rand((M, K), dtype, 91, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 93, 0.1)
    if b_kmajor:
        w = _rand((N, K), dtype, 92, 1 / math.sqrt(K))
        b, bd = w.t(), w.to(DEV).t()
    else:
        b = _rand((K, N), dtype, 92, 1 / math.sqrt(K))
        bd = b.to(DEV)
    c = b2.gemm(a.to(DEV), bd, bias.to(DEV), act, out_dtype, alpha=1.25)
    assert b2.last_kernel() == "gemm_sm100_pair"
    assert c.dtype == out_dtype
    _check(c, O.ref_gemm(a, b, bias, act, torch.float32, alpha=1.25), dtype)
    assert b2.device_status(0) == 0


# Pair launches whose last wave fills at most half the pairs compute those
# tiles as two 256 x 128 halves on two pairs (4096^3: 256 tiles on 74 pairs,
# the 34 left over in halves; 1024 x 5888: 18 left over). Both B layouts and
# ragged M/N/K (the last column tile's second half only partly inside N).
@pytest.mark.parametrize("M,N,K,b_kmajor,out_dtype", [
    (4096, 4096, 4096, False, torch.float16),
    (1024, 5888, 2048, True, torch.bfloat16),
    (1000, 5800, 2104, False, torch.float32),
    (1000, 5800, 2104, True, torch.float16),
])
def test_gemm_pair_last_wave_halves(M, N, K, b_kmajor, out_dtype):
    dtype = torch.bfloat16 if out_dtype == torch.bfloat16 else torch.float16
    a = _rand((M, K), dtype, 95, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 97, 0.1)
    if b_kmajor:
        w = _rand((N, K), dtype, 96, 1 / math.sqrt(K))
        b, bd = w.t(), w.to(DEV).t()
    else:
        b = _rand((K, N), dtype, 96, 1 / math.sqrt(K))
        bd = b.to(DEV)
    c = b2.gemm(a.to(DEV), bd, bias.to(DEV), "relu", out_dtype)
    assert b2.last_kernel() == "gemm_sm100_pair"
    _check(c, O.ref_gemm(a, b, bias, "relu", torch.float32), dtype)
    assert b2.device_status(0) == 0


def test_gemm_epilogue_chain_on_pair_halves():
    """The general epilogue chain on a pair launch whose last wave runs in halves."""
    M, N, K = 2304, 2304, 2048  # 81 tiles on 74 pairs: 7 left over, in halves
    a = _rand((M, K), torch.float16, 98, 1 / math.sqrt(K))
    b = _rand((K, N), torch.float16, 99, 1 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 100, 0.1)
    chain = [("add_bias",), ("mul", 1.5), ("add", -0.25), ("tanh",), ("clamp", -0.5, 0.75)]
    c = b2.gemm_epilogue(a.to(DEV), b.to(DEV), chain, bias.to(DEV), torch.float32)
    assert b2.last_kernel() == "gemm_sm100_pair"
    ref = O.ref_gemm_epilogue(a, b, chain, bias, torch.float32)
    _check(c, ref, torch.float16)


@pytest.mark.parametrize("act", ["none", "relu", "gelu", "silu"])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16])
def test_gemm_splitk_epilogue_and_k_major_b(act, out_dtype):
    M, N, K = 200, 392, 6144
    x = _rand((M, K), torch.bfloat16, 71, 1 / math.sqrt(K))
    w = _rand((N, K), torch.bfloat16, 72, 1 / math.sqrt(K))
    bias = _rand((N,), torch.bfloat16, 73, 0.1)
    c = b2.gemm(x.to(DEV), w.to(DEV).t(), bias.to(DEV), act, out_dtype, alpha=0.75)
    assert b2.last_kernel() == "gemm_sm100_splitk"
    assert c.dtype == out_dtype
    _check(c, O.ref_gemm(x, w.t(), bias, act, torch.float32, alpha=0.75), torch.bfloat16)


def test_gemm_splitk_is_deterministic_and_falls_back_without_workspace():
    from triton_msl_b200 import _lib
    M, N, K = 128, 256, 8192
    a = _rand((M, K), torch.float16, 81, 1 / math.sqrt(K)).to(DEV)
    b = _rand((K, N), torch.float16, 82, 1 / math.sqrt(K)).to(DEV)
    c1, c2 = b2.gemm(a, b), b2.gemm(a, b)
    assert b2.last_kernel() == "gemm_sm100_splitk"
    assert torch.equal(c1, c2)
    L = _lib.lib()
    assert L.b2_query_workspace(0, M, N, K, _lib.B2_F16) > 0
    c3 = torch.empty_like(c1)
    st = L.b2_gemm(a.data_ptr(), b.data_ptr(), None, c3.data_ptr(), M, N, K,
                   _lib.i64_array([K, 1, N, 1, N, 1]), 1.0, 0, _lib.B2_F16, _lib.B2_F32, _lib.B2_F16,
                   None, 0, torch.cuda.current_stream().cuda_stream)
    _lib.check("b2_gemm", st)
    assert L.b2_last_kernel().decode() == "gemm_sm100_n128"
    _check(c3, O.ref_gemm(a.cpu(), b.cpu(), out_dtype=torch.float32), torch.float16)


def test_gemm_k_major_b_linear_layout():
    """x @ w.t() (nn.Linear): B is K-major; still the tensor-core kernel."""
    x = _rand((777, 1024), torch.bfloat16, 51, 1 / 32)
    w = _rand((1536, 1024), torch.bfloat16, 52, 1 / 32)
    bias = _rand((1536,), torch.bfloat16, 53, 0.1)
    c = b2.gemm(x.to(DEV), w.to(DEV).t(), bias.to(DEV), "relu")
    assert b2.last_kernel().startswith("gemm_sm100")
    _check(c, O.ref_gemm(x, w.t(), bias, "relu", torch.float32), torch.bfloat16)


def test_gemm_config3_prime_fp32():
    """fp32 inputs at 2048^3 (benchmark configuration 3'), max-abs 1e-4, on the 3xTF32
    tensor-core path."""
    cfg = W.GEMM_F32
    a, b, _ = W.gemm_inputs(cfg, seed=0)
    c = b2.gemm(a.to(DEV), b.to(DEV))
    assert b2.last_kernel() == "gemm_sm100_tf32x3"
    _check(c, O.ref_gemm(a, b), torch.float32)


def _gemm_no_workspace(a, b, bias=None, act="none"):
    """b2_gemm through the C ABI with no workspace: fp32 takes the FMA path."""
    from triton_msl_b200 import _lib
    c = torch.empty((a.shape[0], b.shape[1]), dtype=torch.float32, device=DEV)
    st = _lib.lib().b2_gemm(a.data_ptr(), b.data_ptr(), bias.data_ptr() if bias is not None else None,
                            c.data_ptr(), a.shape[0], b.shape[1], a.shape[1],
                            _lib.i64_array([*a.stride(), *b.stride(), *c.stride()]), 1.0,
                            _lib.ACT[act], _lib.B2_F32, _lib.B2_F32, _lib.B2_F32, None, 0,
                            torch.cuda.current_stream().cuda_stream)
    _lib.check("b2_gemm", st)
    return c


def test_gemm_fp32_fma_path_without_workspace():
    a = _rand((257, 129), torch.float32, 81)
    b = _rand((129, 95), torch.float32, 82, 1 / math.sqrt(129))
    bias = _rand((95,), torch.float32, 83, 0.1)
    c = _gemm_no_workspace(a.to(DEV), b.to(DEV), bias.to(DEV), "gelu")
    assert b2.last_kernel() == "gemm_simt"
    _check(c, O.ref_gemm(a, b, bias, "gelu"), torch.float32)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (129, 257, 33), (300, 200, 1000), (64, 512, 7),
                                   (1000, 96, 520)])
@pytest.mark.parametrize("b_layout", ["kn", "nk"])
def test_gemm_tf32x3_shapes_layouts(M, N, K, b_layout):
    """3xTF32: ragged M/N/K (K padded per segment), B as [K,N] or a transposed
    [N,K] view (the split pass reads either), max-abs 1e-4 against fp32
    (entries of C ~ N(0, 1))."""
    s4 = K ** -0.25
    a = _rand((M, K), torch.float32, 84, s4)
    if b_layout == "kn":
        b = _rand((K, N), torch.float32, 85, s4).to(DEV)
    else:
        b = _rand((N, K), torch.float32, 85, s4).to(DEV).t()
    bias = _rand((N,), torch.float32, 86, 0.1)
    c = b2.gemm(a.to(DEV), b, bias.to(DEV), "relu")
    assert b2.last_kernel() == "gemm_sm100_tf32x3"
    _check(c, O.ref_gemm(a, b.cpu(), bias, "relu"), torch.float32)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_gemm_tf32x3_low_precision_out(out_dtype):
    a = _rand((200, 300), torch.float32, 87)
    b = _rand((300, 160), torch.float32, 88, 1 / math.sqrt(300))
    c = b2.gemm(a.to(DEV), b.to(DEV), None, "silu", out_dtype)
    assert b2.last_kernel() == "gemm_sm100_tf32x3"
    _check(c, O.ref_gemm(a, b, None, "silu", torch.float32), out_dtype)


@pytest.mark.parametrize("K", [2048, 8192])
def test_gemm_tf32x3_error_growth_with_k(K):
    """The tensor core's fp32 accumulation loses about one unit in the last
    place of the running sum per K=8 step, so the error grows with K and with
    |C| (measured on B200: ~2.7e-5 of max|C| at K=2048, ~1.9e-4 at K=16384),
    an order below plain TF32 and well inside 1e-4 for configs like the benchmark's
    (A, B ~ N(0,1)/sqrt(K), |C| ~ 0.02: 2.3e-6 at 2048^3). Bound written here:
    max-abs <= 5e-5 * (K / 2048) * max|C|."""
    a = _rand((256, K), torch.float32, 89)
    b = _rand((K, 256), torch.float32, 90, 1 / math.sqrt(K))
    ref = a.double() @ b.double()
    c = b2.gemm(a.to(DEV), b.to(DEV)).double().cpu()
    bound = 5e-5 * (K / 2048) * ref.abs().max().item()
    assert (c - ref).abs().max().item() <= bound


def test_gemm_tf32x3_beats_plain_tf32_accuracy():
    """The hi/lo split is what meets 1e-4: plain TF32 (torch with TF32 matmul
    allowed) misses it on this input, 3xTF32 does not."""
    a = _rand((256, 2048), torch.float32, 89)
    b = _rand((2048, 256), torch.float32, 90)
    ref = O.ref_gemm(a, b)
    c = b2.gemm(a.to(DEV), b.to(DEV))
    assert O.max_abs_err(c, ref) <= 0.05  # |C| ~ 180 here
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        plain = a.to(DEV) @ b.to(DEV)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert O.max_abs_err(plain, ref) > 10 * O.max_abs_err(c, ref)


def test_gemm_odd_strides_fall_back_to_cuda_cores():
    a = _rand((130, 70), torch.float16, 61, 0.1)   # K=70: rows not 16-byte pitched
    b = _rand((70, 90), torch.float16, 62, 0.1)
    c = b2.gemm(a.to(DEV), b.to(DEV), activation="relu")
    assert b2.last_kernel() == "gemm_simt"
    _check(c, O.ref_gemm(a, b, None, "relu", torch.float32), torch.float16)


def test_gemm_config3_full_size_sampled():
    """benchmark configuration 3 at full size (8192^3 + bias + ReLU, fp16 out), checked on
    sampled row blocks against the fp32 oracle."""
    cfg = W.GEMM_F16
    a, b, bias = W.gemm_inputs(cfg, device=DEV, seed=0)
    c = b2.gemm(a, b, bias, "relu", torch.float16)
    assert b2.last_kernel().startswith("gemm_sm100")
    for r0 in (0, 4096 - 64, 8192 - 128):
        ref = O.ref_gemm(a[r0:r0 + 128].cpu(), b.cpu(), bias.cpu(), "relu", torch.float32)
        _check(c[r0:r0 + 128], ref, torch.float16)


# ------------------------------------------------------------------- row ops
ROW_OPS = ["softmax", "layernorm", "rmsnorm", "sum", "max", "min", "argmax", "argmin"]


def _row_run(op, x, w, b):
    if op == "softmax":
        return b2.row_softmax(x)
    if op == "layernorm":
        return b2.row_layernorm(x, w, b, 1e-5)
    if op == "rmsnorm":
        return b2.row_rmsnorm(x, w, 1e-6)
    return getattr(b2, f"row_{op}")(x)


def _row_ref(op, x, w, b):
    return O.ROW_REFS[op](x, w, b, 1e-5 if op == "layernorm" else 1e-6)


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(257, 4096), (64, 1000), (33, 4097), (128, 7), (5, 1),
                                       (16, 32768), (4, 40000), (1000, 128)])
def test_row_ops_match_oracle(op, dtype, rows, cols):
    x = _rand((rows, cols), dtype, rows * 7 + cols)
    w = (1 + 0.1 * _rand((cols,), torch.float32, 3)).to(dtype)
    b = (0.1 * _rand((cols,), torch.float32, 4)).to(dtype)
    got = _row_run(op, x.to(DEV), w.to(DEV), b.to(DEV))
    ref = _row_ref(op, x, w, b)
    if op.startswith("arg"):
        assert torch.equal(got.cpu(), ref)
    else:
        _check(got, ref, dtype)


@pytest.mark.parametrize("op", ["sum", "max", "min", "argmax", "argmin"])
def test_row_split_path_long_rows(op):
    x = _rand((3, 1 << 20), torch.float32, 77)
    x[1, 777777] = 9.0
    x[1, 5] = 9.0   # tie: lower index wins
    got = _row_run(op, x.to(DEV), None, None)
    assert b2.last_kernel() == "row_split"
    ref = _row_ref(op, x, None, None)
    if op.startswith("arg"):
        assert torch.equal(got.cpu(), ref)
    elif op == "sum":
        # 1M-element sums: compare against a float64 sum, relative to sum|x|
        exact = x.double().sum(-1)
        assert ((got.cpu().double() - exact).abs() / x.double().abs().sum(-1)).max() < 1e-6
    else:
        assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_row_long_rows_match_oracle(op, dtype):
    """Rows past the register-resident limit (two-pass long-row kernel): row 1
    rises steadily, so the online softmax max grows in every vector and the
    running sum is rescaled throughout; row 2 has a tie for the maximum."""
    rows, cols = 6, 65536 + 24
    x = _rand((rows, cols), torch.float32, 91)
    x[1] = torch.linspace(-20.0, 20.0, cols)
    x[2, 100] = x[2, 60000] = 50.0
    x = x.to(dtype)
    w = (1 + 0.1 * _rand((cols,), torch.float32, 3)).to(dtype)
    b = (0.1 * _rand((cols,), torch.float32, 4)).to(dtype)
    got = _row_run(op, x.to(DEV), w.to(DEV), b.to(DEV))
    ref = _row_ref(op, x, w, b)
    if op.startswith("arg"):
        assert torch.equal(got.cpu(), ref)
    elif op == "sum":
        # 65K-element sums of values up to +-20: against a float64 sum, relative to sum|x|
        exact = x.double().sum(-1)
        err = (got.cpu().double() - exact).abs() / x.double().abs().sum(-1)
        assert err.max() < (1e-6 if dtype == torch.float32 else 4e-3)
    else:
        _check(got, ref, dtype)


def test_row_long_rows_nan_tie_inf():
    x = torch.randn(6, 70000)
    x[0, :] = 2.0                       # all equal: index 0
    x[1, 10] = x[1, 69000] = 99.0       # tie: lower index
    x[2, 50000] = float("nan")          # NaN wins argmax / argmin / max / min
    x[3, 7] = x[3, 65000] = float("nan")
    x[4, :] = float("-inf")
    x[5, :] = float("inf")
    xd = x.to(DEV)
    assert torch.equal(b2.row_argmax(xd).cpu(), O.ref_argmax(x))
    assert torch.equal(b2.row_argmin(xd).cpu(), O.ref_argmin(x))
    assert torch.allclose(b2.row_max(xd).cpu(), O.ref_max(x), equal_nan=True)
    assert torch.allclose(b2.row_min(xd).cpu(), O.ref_min(x), equal_nan=True)
    sm = b2.row_softmax(xd).cpu()
    assert torch.isnan(sm[2]).all() and torch.isnan(sm[4]).all()
    assert torch.allclose(sm[0], torch.full((70000,), 1 / 70000.0), rtol=1e-5)
    assert torch.allclose(sm[1], O.ref_softmax(x[1:2])[0], atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("cols", [8, 1000, 4096, 32768])
def test_row_arg_16bit_ties_nan(dtype, cols):
    """argmax / argmin over fp16 / bf16 rows (values compared two at a time in
    their own type): small integers make ties everywhere (lowest column wins),
    plus NaN (first NaN wins), all -inf and all-equal rows."""
    g = torch.Generator().manual_seed(cols)
    x = torch.randint(-3, 4, (40, cols), generator=g).to(dtype)
    x[1, cols // 2] = float("nan")
    x[2, cols - 1] = float("nan")
    x[2, cols // 3] = float("nan")
    x[3, :] = float("-inf")
    x[4, :] = float("inf")
    x[5, :] = 1.0
    x[6, cols - 1] = 100.0
    xd = x.to(DEV)
    assert torch.equal(b2.row_argmax(xd).cpu(), O.ref_argmax(x))
    assert torch.equal(b2.row_argmin(xd).cpu(), O.ref_argmin(x))


def test_row_nan_and_tie_semantics():
    x = torch.randn(8, 300)
    x[0, :] = 2.0
    x[1, 10] = x[1, 200] = 99.0
    x[2, 123] = float("nan")
    x[3, 7] = x[3, 250] = float("nan")
    x[4, 0] = float("-inf")
    xd = x.to(DEV)
    assert torch.equal(b2.row_argmax(xd).cpu(), O.ref_argmax(x))
    assert torch.equal(b2.row_argmin(xd).cpu(), O.ref_argmin(x))
    assert torch.allclose(b2.row_max(xd).cpu(), O.ref_max(x), equal_nan=True)
    assert torch.allclose(b2.row_min(xd).cpu(), O.ref_min(x), equal_nan=True)
    s = b2.row_sum(xd).cpu()
    assert torch.isnan(s[2]) and torch.isnan(s[3])


def test_row_edge_shapes():
    x = torch.randn(0, 16, device=DEV)
    assert b2.row_softmax(x).shape == (0, 16)
    assert b2.row_sum(torch.randn(4, 0, device=DEV)).tolist() == [0, 0, 0, 0]
    with pytest.raises(b2.B2Error):
        b2.row_argmax(torch.randn(4, 0, device=DEV))
    x3 = torch.randn(2, 3, 96, device=DEV)
    assert torch.allclose(b2.row_softmax(x3).cpu(), O.ref_softmax(x3.cpu()), atol=1e-6)
    xs = torch.randn(64, 200, device=DEV)[:, :100]      # row stride 200
    assert torch.allclose(b2.row_rmsnorm(xs).cpu(), O.ref_rmsnorm(xs.cpu()), atol=1e-5)


def test_row_config4_full_size_properties():
    """benchmark configuration 4 at full size: sampled rows vs the oracle, plus
    size-independent properties over every row."""
    x, w, b = W.row_inputs(W.ROWS_F32, device=DEV, seed=0)
    idx = torch.tensor([0, 1, 4095, 32768, 65535])
    xs = x[idx].cpu()
    sm = b2.row_softmax(x)
    assert ((sm.sum(-1) - 1).abs().max().item()) < 1e-5
    _check(sm[idx], O.ref_softmax(xs), torch.float32)
    ln = b2.row_layernorm(x, w, b, 1e-5)
    _check(ln[idx], O.ref_layernorm(xs, w.cpu(), b.cpu(), 1e-5), torch.float32)
    rn = b2.row_rmsnorm(x, w, 1e-6)
    _check(rn[idx], O.ref_rmsnorm(xs, w.cpu(), 1e-6), torch.float32)
    am = b2.row_argmax(x)
    assert torch.equal(am, torch.argmax(x, dim=-1))
    mx = b2.row_max(x)
    assert torch.equal(mx, x.gather(1, am[:, None])[:, 0])
    _check(b2.row_sum(x)[idx], O.ref_sum(xs), torch.float32)


def test_device_status_clean():
    assert b2.device_status(0) == 0


@pytest.mark.parametrize("D", [128, 64, 32])
def test_fa_config2_full_size_sampled(D):
    """benchmark configuration 2 at full size ([4,16,2048,D] fp16 causal, N(0,1)*0.5),
    checked on sampled (batch, head) slices against the oracle."""
    cfg = W.FAConfig("c2", 4, 16, 2048, D, True, torch.float16, 0.5)
    q, k, v = W.fa_inputs(cfg, device=DEV, seed=0)
    o = b2.flash_attn_fwd(q, k, v, causal=True)
    assert b2.last_kernel() == "fa_sm100"
    for bb, hh in ((0, 0), (1, 7), (3, 15)):
        sl = (slice(bb, bb + 1), slice(hh, hh + 1))
        ref = O.ref_attention(q[sl].cpu(), k[sl].cpu(), v[sl].cpu(), True)
        _check(o[sl], ref, torch.float16)


def test_fa_config5_full_size_sampled():
    """benchmark configuration 5 attention at full size ([64,32,8192,128] bf16 causal),
    sampled heads against the oracle plus a finiteness check over all of O."""
    cfg = W.FA_BF16_SCALE
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = ((torch.randn((cfg.B, cfg.H, cfg.S, cfg.D), generator=g, device=DEV) * cfg.std)
               .to(cfg.dtype) for _ in range(3))
    o = b2.flash_attn_fwd(q, k, v, causal=True)
    assert b2.last_kernel() == "fa_sm100"
    assert torch.isfinite(o).all()
    for bb, hh in ((0, 0), (63, 31)):
        sl = (slice(bb, bb + 1), slice(hh, hh + 1))
        ref = O.ref_attention(q[sl].cpu(), k[sl].cpu(), v[sl].cpu(), True)
        _check(o[sl], ref, torch.bfloat16)


def test_gemm_config5_full_size_sampled():
    """benchmark configuration 5 GEMM at full size (65536 x 16384 x 16384 bf16), sampled
    row blocks against the fp32 oracle."""
    cfg = W.GEMM_BF16_SCALE
    a, b, _ = W.gemm_inputs(cfg, device=DEV, seed=0)
    c = b2.gemm(a, b)
    assert b2.last_kernel().startswith("gemm_sm100")
    for r0 in (0, 32768 + 64, 65536 - 128):
        ref = O.ref_gemm(a[r0:r0 + 128].cpu(), b.cpu(), out_dtype=torch.float32)
        _check(c[r0:r0 + 128], ref, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(512, 256, 512), (300, 200, 136), (128, 64, 64)])
def test_gemm_softmax_epilogue(dtype, M, N, K):
    """Fused matmul -> row softmax (reference _lowerer_templates.py:1515-1728)."""
    a = _rand((M, K), dtype, 71, 1.0)
    b = _rand((K, N), dtype, 72, 1.0 / math.sqrt(K))
    bias = _rand((N,), torch.float32, 73, 0.3)
    c = b2.gemm(a.to(DEV), b.to(DEV), bias.to(DEV), "softmax", torch.float32)
    assert b2.last_kernel().startswith("gemm_sm100")
    ref = O.ref_gemm(a, b, bias, "softmax", torch.float32)
    _check(c, ref, dtype)
    assert (c.sum(-1) - 1).abs().max().item() < 1e-4


def test_gemm_softmax_epilogue_fp32_and_limits():
    a = _rand((100, 64), torch.float32, 74)
    b = _rand((64, 96), torch.float32, 75, 0.125)
    c = b2.gemm(a.to(DEV), b.to(DEV), None, "softmax")
    assert b2.last_kernel() == "gemm_sm100_tf32x3"
    _check(c, O.ref_gemm(a, b, None, "softmax"), torch.float32)
    c = _gemm_no_workspace(a.to(DEV), b.to(DEV), None, "softmax")
    assert b2.last_kernel() == "gemm_simt+row_softmax"
    _check(c, O.ref_gemm(a, b, None, "softmax"), torch.float32)
    with pytest.raises(b2.B2Unsupported):
        b2.gemm(a.to(DEV), _rand((64, 300), torch.float32, 76).to(DEV), None, "softmax")


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("chunks", [None, 1, 3, 64])
def test_fa_host_pipeline_matches_device_path(causal, chunks):
    """flash_attn_fwd_host (host tensors, copies overlapped with the kernel per
    (batch, head) chunk) returns exactly what the device entry point returns."""
    q, k, v = (_rand((2, 5, 300, 64), torch.float16, s, 0.5).pin_memory() for s in (91, 92, 93))
    o = b2.flash_attn_fwd_host(q, k, v, causal=causal, chunks=chunks)
    torch.cuda.synchronize()
    assert not o.is_cuda
    ref = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal).cpu()
    assert torch.equal(o, ref)
    _check(o, O.ref_attention(q, k, v, causal), torch.float16)


@pytest.mark.parametrize("ready", [False, True])
def test_fa_host_pipeline_back_to_back_calls_reuse_staging(ready):
    """Calls queued without synchronising, with inputs that grow and shrink: the
    two device staging slots are reused (and regrown) only after the call that
    last used them has read its output back, so every output is intact; with
    host_inputs_ready the uploads of one call overlap the previous read-back."""
    shapes = [(1, 4, 256, 64), (2, 6, 300, 64), (1, 3, 128, 128), (2, 8, 512, 64), (1, 2, 64, 32),
              (2, 8, 512, 64), (1, 4, 256, 64)]
    cases = []
    for i, shp in enumerate(shapes):
        q, k, v = (_rand(shp, torch.float16, 200 + 3 * i + s, 0.5).pin_memory() for s in range(3))
        cases.append((q, k, v, b2.flash_attn_fwd_host(q, k, v, causal=bool(i & 1),
                                                      chunks=3 if i % 3 else None,
                                                      host_inputs_ready=ready)))
    torch.cuda.synchronize()
    for i, (q, k, v, o) in enumerate(cases):
        ref = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=bool(i & 1)).cpu()
        assert torch.equal(o, ref), f"call {i}"
    b2.host_pipeline.release_staging()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_fa_many_units_per_cta_and_rescales(dtype, D, causal):
    """More (query block, head) units than SMs, so each persistent CTA runs several
    units of different lengths back to back (per-tile O / Q hand-over between
    units), with scores spread wide enough (x3 inputs) that the running max grows
    by more than 2^8 mid-row and the O rescale path runs."""
    q, k, v = (_rand((4, 50, 384, D), dtype, s, 1.5) for s in (94, 95, 96))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    assert b2.last_kernel() == "fa_sm100"
    _check(o, O.ref_attention(q, k, v, causal), dtype)
    assert b2.device_status(0) == 0


@pytest.mark.parametrize("D", [32, 128])
@pytest.mark.parametrize("S", [1, 2, 8])
@pytest.mark.parametrize("causal", [False, True])
def test_fa_tiny_sequences(S, causal, D):
    q, k, v = (_rand((3, 4, S, D), torch.float16, s, 0.5) for s in (97, 98, 99))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    assert b2.last_kernel() == "fa_sm100"
    _check(o, O.ref_attention(q, k, v, causal), torch.float16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_fa_rescale_when_later_keys_dominate(dtype, D, causal):
    """Keys of later blocks score far higher than the first block's, so the
    running max grows by more than 2^8 after the first block and O (and l) are
    rescaled mid-row. For D <= 64 l is accumulated by the tensor core beside O,
    so this also checks its rescale."""
    q = _rand((2, 3, 640, D), torch.float32, 101, 1.0)
    k = _rand((2, 3, 640, D), torch.float32, 102, 1.0)
    k[:, :, 256:] *= 5.0
    v = _rand((2, 3, 640, D), torch.float32, 103, 1.0)
    q, k, v = (t.to(dtype) for t in (q, k, v))
    o = b2.flash_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    assert b2.last_kernel() == "fa_sm100"
    _check(o, O.ref_attention(q, k, v, causal), dtype)
