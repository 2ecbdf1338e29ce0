"""PyTorch operator surface of the hot path, registered as torch.library custom ops.

Operators (namespace ``b2msl``):
  * ``flash_attn_fwd(q, k, v, causal, sm_scale) -> o``       q/k/v/o: [B, H, S, D]
  * ``gemm(a, b, bias, activation, out_dtype, alpha) -> c``  c = act(alpha*a@b + bias)
  * ``row_softmax / row_layernorm / row_rmsnorm (x[..., cols]) -> like x``
  * ``row_sum / row_max / row_min (x) -> x.shape[:-1]`` and
    ``row_argmax / row_argmin (x) -> int64 x.shape[:-1]``

They replace, for this path, what the reference produces from @triton.jit
kernels through its Metal templates (FA: tests/test_flash_attention.py:35-118
-> _msl_templates.py:1833-2070; matmul: tests/test_fast_matmul_parity.py:14-27
-> _msl_templates.py:4134-4255 + _lowerer_templates.py:1515-1855; rows:
_lowerer_templates.py:992-1320, _lowerer_reduce.py:773-1333). Each op is a
thin wrapper over one C-ABI call on the tensors' device and current stream.
Inputs must be CUDA tensors; anything else raises (no CPU fallback).
"""
from __future__ import annotations

import math
import ctypes
from typing import List, Optional, Sequence

import torch

from . import _lib

_DT = {torch.float32: _lib.B2_F32, torch.float16: _lib.B2_F16, torch.bfloat16: _lib.B2_BF16}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: unsupported dtype {t.dtype} (float32/float16/bfloat16)") from None


def _require_cuda(*ts: Optional[torch.Tensor], what: str) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{what}: tensors must be on a CUDA device (got {t.device}); "
                               "b2msl has no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on different devices ({dev} vs {t.device})")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


# ------------------------------------------------------------------ attention
def _fa_impl(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
             sm_scale: float) -> torch.Tensor:
    what = "flash_attn_fwd"
    dev = _require_cuda(q, k, v, what=what)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"{what}: q, k, v must all be [B, H, S, D] of one shape; got "
                         f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"{what}: q, k, v must share a dtype")
    o = torch.empty(tuple(q.shape), dtype=q.dtype, device=dev)
    _fa_into(q, k, v, o, causal, sm_scale, _stream(dev))
    return o


def _fa_into(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, causal: bool,
             sm_scale: float, stream: int) -> None:
    """b2_fa_fwd into a caller-owned o (same shape as q) on the CUDA stream handle `stream`."""
    dt = _dtype_code(q, "flash_attn_fwd")
    B, H, S, D = q.shape
    strides = [*q.stride(), *k.stride(), *v.stride(), *o.stride()]
    with torch.cuda.device(q.device):
        st = _lib.lib().b2_fa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                  B, H, S, D, _lib.i64_array(strides), float(sm_scale),
                                  1 if causal else 0, dt, stream)
    _lib.check("b2_fa_fwd", st)


@torch.library.custom_op("b2msl::flash_attn_fwd", mutates_args=())
def _fa_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
           sm_scale: float) -> torch.Tensor:
    return _fa_impl(q, k, v, causal, sm_scale)


@_fa_op.register_fake
def _(q, k, v, causal, sm_scale):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


def flash_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   sm_scale: Optional[float] = None) -> torch.Tensor:
    """o = softmax(sm_scale * q @ k^T [causal]) @ v over [B, H, S, D] tensors.

    sm_scale defaults to 1/sqrt(D), the scale the reference kernel bakes in
    (tests/test_flash_attention.py:63-65).
    """
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    return torch.ops.b2msl.flash_attn_fwd(q, k, v, bool(causal), float(sm_scale))


# ---------------------------------------------------------------------- gemm
def _gemm_impl(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], activation: str,
               out_dtype: Optional[torch.dtype], alpha: float) -> torch.Tensor:
    what = "gemm"
    dev = _require_cuda(a, b, bias, what=what)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"{what}: need a[M,K] @ b[K,N]; got {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != b.dtype:
        raise TypeError(f"{what}: a and b must share a dtype ({a.dtype} vs {b.dtype})")
    if activation not in _lib.ACT:
        raise ValueError(f"{what}: activation must be one of {sorted(_lib.ACT)}")
    M, K = a.shape
    N = b.shape[1]
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != N):
        raise ValueError(f"{what}: bias must be [N={N}]")
    odt = out_dtype or a.dtype
    c = torch.empty((M, N), dtype=odt, device=dev)
    cout = _dtype_code(c, what)
    bdt = _dtype_code(bias, what) if bias is not None else _lib.B2_F32
    strides = [a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1)]
    L = _lib.lib()
    with torch.cuda.device(dev):
        # fp32 inputs run as 3xTF32 on the tensor cores with this scratch
        ws_bytes = L.b2_query_workspace(0, M, N, K, _dtype_code(a, what))
        ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev) if ws_bytes else None
        st = L.b2_gemm(a.data_ptr(), b.data_ptr(),
                       bias.data_ptr() if bias is not None else None, c.data_ptr(),
                       M, N, K, _lib.i64_array(strides), float(alpha),
                       _lib.ACT[activation], _dtype_code(a, what), bdt, cout,
                       ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    _lib.check("b2_gemm", st)
    return c


@torch.library.custom_op("b2msl::gemm", mutates_args=())
def _gemm_op(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], activation: str,
             out_dtype: Optional[torch.dtype], alpha: float) -> torch.Tensor:
    return _gemm_impl(a, b, bias, activation, out_dtype, alpha)


@_gemm_op.register_fake
def _(a, b, bias, activation, out_dtype, alpha):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype or a.dtype)


def gemm(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor] = None,
         activation: str = "none", out_dtype: Optional[torch.dtype] = None,
         alpha: float = 1.0) -> torch.Tensor:
    """c = activation(alpha * (a @ b) + bias[None, :]) with fp32 accumulation.

    activation: none / relu / gelu / gelu_tanh / silu, or softmax (a softmax over
    each output row, the reference's fused matmul + row-softmax; N <= 256).
    """
    return torch.ops.b2msl.gemm(a, b, bias, activation, out_dtype, float(alpha))


def _epi_program(ops):
    """[(name, *constants)] -> (codes, args) for b2_gemm_epilogue."""
    codes, args = [], []
    for op in ops:
        name, consts = op[0], [float(c) for c in op[1:]]
        if name not in _lib.EPI:
            raise ValueError(f"gemm_epilogue: unknown op {name!r} (one of {sorted(_lib.EPI)})")
        code, n = _lib.EPI[name]
        if len(consts) != n:
            raise ValueError(f"gemm_epilogue: op {name!r} takes {n} constant(s), got {len(consts)}")
        codes.append(code)
        args += (consts + [0.0, 0.0])[:2]
    if len(codes) > _lib.EPI_MAX_OPS:
        raise ValueError(f"gemm_epilogue: at most {_lib.EPI_MAX_OPS} ops")
    return codes, args


def _gemm_epi_impl(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], codes: List[int],
                   args: List[float], out_dtype: Optional[torch.dtype]) -> torch.Tensor:
    what = "gemm_epilogue"
    dev = _require_cuda(a, b, bias, what=what)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"{what}: need a[M,K] @ b[K,N]; got {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != b.dtype:
        raise TypeError(f"{what}: a and b must share a dtype ({a.dtype} vs {b.dtype})")
    M, K = a.shape
    N = b.shape[1]
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != N):
        raise ValueError(f"{what}: bias must be [N={N}]")
    c = torch.empty((M, N), dtype=out_dtype or a.dtype, device=dev)
    strides = [a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1)]
    n = len(codes)
    codes_c = (ctypes.c_int32 * max(n, 1))(*codes)
    args_c = (ctypes.c_float * max(2 * n, 2))(*args)
    L = _lib.lib()
    with torch.cuda.device(dev):
        ws_bytes = L.b2_query_workspace(0, M, N, K, _dtype_code(a, what))
        ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev) if ws_bytes else None
        st = L.b2_gemm_epilogue(a.data_ptr(), b.data_ptr(),
                                bias.data_ptr() if bias is not None else None, c.data_ptr(),
                                M, N, K, _lib.i64_array(strides), codes_c, args_c, n,
                                _dtype_code(a, what),
                                _dtype_code(bias, what) if bias is not None else _lib.B2_F32,
                                _dtype_code(c, what), ws.data_ptr() if ws is not None else None,
                                ws_bytes, _stream(dev))
    _lib.check("b2_gemm_epilogue", st)
    return c


@torch.library.custom_op("b2msl::gemm_epilogue", mutates_args=())
def _gemm_epi_op(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], codes: List[int],
                 args: List[float], out_dtype: Optional[torch.dtype]) -> torch.Tensor:
    return _gemm_epi_impl(a, b, bias, codes, args, out_dtype)


@_gemm_epi_op.register_fake
def _(a, b, bias, codes, args, out_dtype):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype or a.dtype)


def gemm_epilogue(a: torch.Tensor, b: torch.Tensor, ops: Sequence[tuple],
                  bias: Optional[torch.Tensor] = None,
                  out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """c = f_n(...f_1(a @ b)) with fp32 math: a general fused epilogue chain.

    ops: sequence of (name, *constants), applied in order to each output
    element, e.g. [("add_bias",), ("mul", 0.5), ("clamp", -1.0, 1.0), ("exp",)].
    Names: add sub rsub mul div rdiv (one constant), add_bias mul_bias (bias[n]),
    max min (NaN-propagating) maxnum minnum (NaN-quiet), clamp clampnum (two),
    neg exp exp2 log log2 sqrt rsqrt sin cos erf tanh floor ceil abs relu gelu
    gelu_tanh silu sigmoid, fma (x * c0 + c1). The reference lowers such chains
    for single-strip matmuls only (_lowerer_templates.py:1749-1855).
    """
    codes, args = _epi_program(ops)
    return torch.ops.b2msl.gemm_epilogue(a, b, bias, codes, args, out_dtype)


# ---------------------------------------------------------------- row family
def _as_rows(x: torch.Tensor) -> torch.Tensor:
    if x.dim() == 0:
        raise ValueError("row ops need at least one dimension")
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.shape[-1] > 0 and x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _row_call(op: str, x: torch.Tensor, w: Optional[torch.Tensor], b: Optional[torch.Tensor],
              eps: float) -> torch.Tensor:
    what = f"row_{op}"
    dev = _require_cuda(x, w, b, what=what)
    dt = _dtype_code(x, what)
    cols = x.shape[-1] if x.dim() else 0
    for p, name in ((w, "weight"), (b, "bias")):
        if p is not None:
            if p.dtype != x.dtype or p.shape != (cols,):
                raise ValueError(f"{what}: {name} must be [{cols}] of dtype {x.dtype}")
            if not p.is_contiguous():
                raise ValueError(f"{what}: {name} must be contiguous")
    x2 = _as_rows(x)
    rows = x2.shape[0]
    row_out = op in ("softmax", "layernorm", "rmsnorm")
    if row_out:
        out = torch.empty((rows, cols), dtype=x.dtype, device=dev)
        ld_out = out.stride(0) if rows else cols
    else:
        odt = torch.int64 if op.startswith("arg") else x.dtype
        out = torch.empty((rows,), dtype=odt, device=dev)
        ld_out = 1
    code = _lib.ROW_OPS[op]
    L = _lib.lib()
    ws_bytes = L.b2_query_workspace(1, code, rows, cols, dt)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev) if ws_bytes else None
    ld_x = x2.stride(0) if rows > 1 else max(cols, 1)
    with torch.cuda.device(dev):
        st = L.b2_row_op(code, x2.data_ptr(), w.data_ptr() if w is not None else None,
                         b.data_ptr() if b is not None else None, out.data_ptr(), rows, cols,
                         ld_x, ld_out, float(eps), dt,
                         ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    _lib.check("b2_row_op", st)
    return out.reshape(x.shape) if row_out else out.reshape(x.shape[:-1])


@torch.library.custom_op("b2msl::row_op", mutates_args=())
def _row_op(x: torch.Tensor, op: str, weight: Optional[torch.Tensor],
            bias: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    return _row_call(op, x, weight, bias, eps)


@_row_op.register_fake
def _(x, op, weight, bias, eps):
    if op in ("softmax", "layernorm", "rmsnorm"):
        return torch.empty_like(x, memory_format=torch.contiguous_format)
    odt = torch.int64 if op.startswith("arg") else x.dtype
    return x.new_empty(x.shape[:-1], dtype=odt)


def row_softmax(x: torch.Tensor) -> torch.Tensor:
    """softmax over the last dimension (reference: tests/test_integration.py:552)."""
    return torch.ops.b2msl.row_op(x, "softmax", None, None, 0.0)


def row_layernorm(x: torch.Tensor, weight: Optional[torch.Tensor] = None,
                  bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """(x - mean) * rsqrt(var + eps) * weight + bias over the last dimension."""
    return torch.ops.b2msl.row_op(x, "layernorm", weight, bias, float(eps))


def row_rmsnorm(x: torch.Tensor, weight: Optional[torch.Tensor] = None,
                eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * weight over the last dimension."""
    return torch.ops.b2msl.row_op(x, "rmsnorm", weight, None, float(eps))


def row_sum(x: torch.Tensor) -> torch.Tensor:
    return torch.ops.b2msl.row_op(x, "sum", None, None, 0.0)


def row_max(x: torch.Tensor) -> torch.Tensor:
    return torch.ops.b2msl.row_op(x, "max", None, None, 0.0)


def row_min(x: torch.Tensor) -> torch.Tensor:
    return torch.ops.b2msl.row_op(x, "min", None, None, 0.0)


def row_argmax(x: torch.Tensor) -> torch.Tensor:
    """int64 index of the row maximum; ties -> lowest index, NaN counts as maximum."""
    return torch.ops.b2msl.row_op(x, "argmax", None, None, 0.0)


def row_argmin(x: torch.Tensor) -> torch.Tensor:
    return torch.ops.b2msl.row_op(x, "argmin", None, None, 0.0)


# ------------------------------------------------------------ any-axis reduce
def _reduce_impl(x: torch.Tensor, op: str, dim: int) -> torch.Tensor:
    what = "reduce"
    dev = _require_cuda(x, what=what)
    if op not in ("sum", "max", "min", "argmax", "argmin"):
        raise ValueError(f"{what}: op must be sum/max/min/argmax/argmin, got {op!r}")
    if x.dim() == 0:
        raise ValueError(f"{what}: needs at least one dimension")
    d = dim % x.dim()
    if d == x.dim() - 1:
        return _row_call(op, x, None, None, 0.0)
    xc = x.contiguous()
    shape = list(x.shape)
    outer = math.prod(shape[:d])
    R = shape[d]
    inner = math.prod(shape[d + 1:])
    out_shape = shape[:d] + shape[d + 1:]
    odt = torch.int64 if op.startswith("arg") else x.dtype
    out = torch.empty(out_shape, dtype=odt, device=dev)
    dt = _dtype_code(x, what)
    L = _lib.lib()
    with torch.cuda.device(dev):
        ws_bytes = L.b2_query_workspace(3, outer, R, inner, 0)
        ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev) if ws_bytes else None
        st = L.b2_reduce_axis(_lib.ROW_OPS[op], xc.data_ptr(), out.data_ptr(), outer, R, inner, dt,
                              ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    _lib.check("b2_reduce_axis", st)
    return out


@torch.library.custom_op("b2msl::reduce", mutates_args=())
def _reduce_op(x: torch.Tensor, op: str, dim: int) -> torch.Tensor:
    return _reduce_impl(x, op, dim)


@_reduce_op.register_fake
def _(x, op, dim):
    d = dim % x.dim()
    shape = list(x.shape[:d]) + list(x.shape[d + 1:])
    return x.new_empty(shape, dtype=torch.int64 if op.startswith("arg") else x.dtype)


def reduce(x: torch.Tensor, op: str, dim: int = -1) -> torch.Tensor:
    """sum / max / min / argmax / argmin of x along `dim` (any axis; keepdim=False).

    The last axis runs the row kernels; another axis runs the middle-axis kernel
    over x viewed as [outer, size(dim), inner] (the reference's generic reduce,
    fuzzed on 2-D and 3-D inputs along axis 0, tests/test_fuzz_reduce.py:88-139).
    argmax/argmin return int64 with ties to the lower index and NaN as extreme.
    """
    return torch.ops.b2msl.reduce(x, op, int(dim))
