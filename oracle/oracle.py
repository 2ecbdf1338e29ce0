"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline;
the product path (triton_msl_b200) never calls it.

It restates, in fp32 torch-CPU arithmetic, the oracle functions the reference
(bledden/triton-msl) uses in its own tests; the reference kernels themselves are
Metal Shading Language and cannot run off Apple hardware. Each function cites
the reference lines it follows. Parity pinning: tests/golden/make_golden.py
imports the reference's own oracle functions from its test modules and records
their outputs on seeded inputs; tests/test_oracle.py checks this module against
those fixtures.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def ref_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                  sm_scale: Optional[float] = None) -> torch.Tensor:
    """softmax((q*scale) @ k^T [tril mask]) @ v in fp32; fully masked rows -> 0.

    Follows tests/test_flash_attention.py:124-135 (`_ref_attention`: q scaled
    before the matmul, tril causal mask, softmax, nan_to_num(nan=0), @ v) with
    the fp16/bf16 upcast of tests/test_fa_simdgroup_diff.py:18-24 (`_ref`).
    """
    qf, kf, vf = q.float(), k.float(), v.float()
    scale = (1.0 / math.sqrt(qf.shape[-1])) if sm_scale is None else float(sm_scale)
    attn = torch.matmul(qf * scale, kf.transpose(-2, -1))
    if causal:
        n = attn.shape[-1]
        mask = torch.tril(torch.ones(n, n))
        attn = attn.masked_fill(mask[None, None] == 0, float("-inf"))
    attn = torch.softmax(attn, dim=-1)
    attn = torch.nan_to_num(attn, nan=0.0)
    return torch.matmul(attn, vf)


def ref_gemm(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor] = None,
             activation: str = "none", out_dtype: Optional[torch.dtype] = None,
             alpha: float = 1.0) -> torch.Tensor:
    """act(alpha * A.float() @ B.float() + bias[None, :]) then cast.

    A.float() @ B.float(): tests/test_fast_matmul_parity.py:53; bias + ReLU:
    tests/test_matmul_epilogue.py:80 (np.maximum(a@b + bias[None,:], 0)); the
    fp16 output cast: tests/test_fast_matmul_parity.py:94 (`.half()`).
    """
    c = a.float() @ b.float()
    if alpha != 1.0:
        c = c * alpha
    if bias is not None:
        c = c + bias.float()[None, :]
    if activation == "relu":
        c = torch.relu(c)
    elif activation == "gelu":
        c = torch.nn.functional.gelu(c)
    elif activation == "gelu_tanh":
        c = torch.nn.functional.gelu(c, approximate="tanh")
    elif activation == "silu":
        c = torch.nn.functional.silu(c)
    elif activation == "softmax":
        # fused matmul -> row softmax (reference _lowerer_templates.py:1515-1728,
        # checked there against torch.softmax(a @ b, dim=1))
        c = torch.softmax(c, dim=-1)
    elif activation != "none":
        raise ValueError(activation)
    return c.to(out_dtype or a.dtype)


def ref_gemm_epilogue(a: torch.Tensor, b: torch.Tensor, ops, bias: Optional[torch.Tensor] = None,
                      out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """A.float() @ B.float() (tests/test_fast_matmul_parity.py:53), then the op
    chain in order in fp32, then the cast. Op meanings follow the reference's
    fused-epilogue tables (triton_msl/codegen/_lowerer_templates.py:1733-1748):
    max/min propagate NaN (arith.maximumf / minimumf), maxnum/minnum are
    NaN-quiet (arith.maxnumf / minnumf); clamp propagates NaN like torch.clamp.
    """
    x = a.float() @ b.float()
    bf = bias.float()[None, :] if bias is not None else None
    for op in ops:
        n, c = op[0], [float(v) for v in op[1:]]
        if n == "add": x = x + c[0]
        elif n == "sub": x = x - c[0]
        elif n == "rsub": x = c[0] - x
        elif n == "mul": x = x * c[0]
        elif n == "div": x = x / c[0]
        elif n == "rdiv": x = c[0] / x
        elif n == "add_bias": x = x + bf
        elif n == "mul_bias": x = x * bf
        elif n == "max": x = torch.maximum(x, torch.tensor(c[0]))
        elif n == "min": x = torch.minimum(x, torch.tensor(c[0]))
        elif n == "maxnum": x = torch.fmax(x, torch.tensor(c[0]))
        elif n == "minnum": x = torch.fmin(x, torch.tensor(c[0]))
        elif n == "clamp": x = torch.clamp(x, c[0], c[1])
        elif n == "clampnum": x = torch.fmin(torch.fmax(x, torch.tensor(c[0])), torch.tensor(c[1]))
        elif n == "neg": x = -x
        elif n == "exp": x = torch.exp(x)
        elif n == "exp2": x = torch.exp2(x)
        elif n == "log": x = torch.log(x)
        elif n == "log2": x = torch.log2(x)
        elif n == "sqrt": x = torch.sqrt(x)
        elif n == "rsqrt": x = torch.rsqrt(x)
        elif n == "sin": x = torch.sin(x)
        elif n == "cos": x = torch.cos(x)
        elif n == "erf": x = torch.erf(x)
        elif n == "tanh": x = torch.tanh(x)
        elif n == "floor": x = torch.floor(x)
        elif n == "ceil": x = torch.ceil(x)
        elif n == "abs": x = torch.abs(x)
        elif n == "relu": x = torch.relu(x)
        elif n == "gelu": x = torch.nn.functional.gelu(x)
        elif n == "gelu_tanh": x = torch.nn.functional.gelu(x, approximate="tanh")
        elif n == "silu": x = torch.nn.functional.silu(x)
        elif n == "sigmoid": x = torch.sigmoid(x)
        elif n == "fma": x = x * c[0] + c[1]
        else:
            raise ValueError(n)
    return x.to(out_dtype or a.dtype)


def ref_softmax(x: torch.Tensor) -> torch.Tensor:
    """torch.softmax(x, dim=-1) in fp32 (tests/test_integration.py:552)."""
    return torch.softmax(x.float(), dim=-1)


def ref_layernorm(x: torch.Tensor, w: Optional[torch.Tensor] = None,
                  b: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """torch.layer_norm over the last dim (tests/test_integration.py:1124)."""
    return torch.layer_norm(x.float(), [x.shape[-1]], None if w is None else w.float(),
                            None if b is None else b.float(), eps)


def ref_rmsnorm(x: torch.Tensor, w: Optional[torch.Tensor] = None,
                eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(mean(x^2) + eps) * w (tests/test_integration.py:1081-1082)."""
    xf = x.float()
    y = xf / torch.sqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)
    return y * w.float() if w is not None else y


def ref_sum(x: torch.Tensor) -> torch.Tensor:
    """A.float().sum(1) (tests/test_fuzz_reduce.py:117-139)."""
    return x.float().sum(-1)


def ref_max(x: torch.Tensor) -> torch.Tensor:
    """A.float().max(1).values (tests/test_fuzz_reduce.py:117-139)."""
    return x.float().max(-1).values


def ref_min(x: torch.Tensor) -> torch.Tensor:
    return x.float().min(-1).values


def ref_argmax(x: torch.Tensor) -> torch.Tensor:
    """A.float().argmax(1), int64 (tests/test_fuzz_reduce.py:131)."""
    return x.float().argmax(-1)


def ref_argmin(x: torch.Tensor) -> torch.Tensor:
    return x.float().argmin(-1)


def ref_reduce_axis(x: torch.Tensor, op: str, dim: int) -> torch.Tensor:
    """A.float().sum(dim) / .max(dim).values / .min(dim).values / .argmax(dim) /
    .argmin(dim) (tests/test_fuzz_reduce.py:88-139: 2d_sum_ax0, 3d_sum_ax0)."""
    xf = x.float()
    if op == "sum":
        return xf.sum(dim)
    if op == "max":
        return xf.max(dim).values
    if op == "min":
        return xf.min(dim).values
    if op == "argmax":
        return xf.argmax(dim)
    if op == "argmin":
        return xf.argmin(dim)
    raise ValueError(op)


ROW_REFS = {
    "softmax": lambda x, w, b, eps: ref_softmax(x),
    "layernorm": lambda x, w, b, eps: ref_layernorm(x, w, b, eps),
    "rmsnorm": lambda x, w, b, eps: ref_rmsnorm(x, w, eps),
    "sum": lambda x, w, b, eps: ref_sum(x),
    "max": lambda x, w, b, eps: ref_max(x),
    "min": lambda x, w, b, eps: ref_min(x),
    "argmax": lambda x, w, b, eps: ref_argmax(x),
    "argmin": lambda x, w, b, eps: ref_argmin(x),
}


# ----------------------------------------------------------- tolerance checks
def normwise_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max|got - ref| / max(max|ref|, 1e-6): the err <= atol + rtol*scale form of
    tests/test_fuzz_reduce.py:207-211 with the scale factored out."""
    g, r = got.detach().float().cpu(), ref.detach().float().cpu()
    return (g - r).abs().max().item() / max(r.abs().max().item(), 1e-6)


def max_abs_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    return (got.detach().float().cpu() - ref.detach().float().cpu()).abs().max().item()


# Tolerances the target states: fp32 paths max-abs <= 1e-4; fp16/bf16 paths
# normwise-relative <= 2e-3; indices bit-exact.
TOL_F32_ABS = 1e-4
TOL_LOWP_REL = 2e-3
