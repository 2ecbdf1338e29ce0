"""triton_msl_b200 — B200 (sm_100a) hot path of triton-msl.

FlashAttention forward, GEMM with bias/activation epilogue and the
row-reduction family, as hand-written CUDA kernels behind a C ABI
(``libb2msl.so``, declared in include/b2msl.h) and exposed as PyTorch custom
ops plus a ``torch.compile`` backend (``backend="b2msl"``).
"""
from ._lib import B2Error, B2Unsupported, last_kernel, device_status  # noqa: F401
from .ops import (  # noqa: F401
    flash_attn_fwd, gemm, gemm_epilogue, row_softmax, row_layernorm, row_rmsnorm, row_sum, row_max,
    row_min, row_argmax, row_argmin, reduce,
)
from .host_pipeline import flash_attn_fwd_host  # noqa: F401

from . import compile_backend as _cb

_cb.register()  # torch.compile(..., backend="b2msl")

__version__ = "0.1.0"
