"""Seeded synthetic inputs for the benchmark configurations of the hot path.

The reference quotes no dataset; its configs are random tensors of stated
shapes and distributions. Generation runs on the CPU with a seeded
torch.Generator (so every process and the CPU baseline see identical values)
or, for full-size inputs, on the device with a seeded CUDA generator.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class FAConfig:
    name: str
    B: int
    H: int
    S: int
    D: int
    causal: bool
    dtype: torch.dtype
    std: float = 1.0

    def flops(self) -> float:
        """Algorithmic FLOPs: 4*B*H*S^2*D, halved for causal (2*B*H*S^2*D)."""
        f = 4.0 * self.B * self.H * self.S * self.S * self.D
        return f / 2 if self.causal else f


@dataclass(frozen=True)
class GemmConfig:
    name: str
    M: int
    N: int
    K: int
    dtype: torch.dtype
    bias: bool
    activation: str
    out_dtype: torch.dtype

    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K


@dataclass(frozen=True)
class RowConfig:
    name: str
    rows: int
    cols: int
    dtype: torch.dtype

    def bytes(self, op: str) -> float:
        """Algorithmic HBM bytes: read X once, write Y (row ops) or one value per row."""
        es = torch.tensor([], dtype=self.dtype).element_size()
        x = self.rows * self.cols * es
        if op in ("softmax", "layernorm", "rmsnorm"):
            params = {"softmax": 0, "layernorm": 2, "rmsnorm": 1}[op] * self.cols * es
            return 2.0 * x + params
        if op.startswith("arg"):
            return x + 8.0 * self.rows
        return x + es * self.rows


# Benchmark configurations of the hot path (numbered as in bench.py and the
# tests): 1 FA fp32 [1,4,256,64]; 2 FA fp16 causal [4,16,2048,D], D = 128 / 64
# / 32; 3 GEMM fp16 8192^3 + bias + ReLU, and 3' fp32 2048^3; 4 the row family
# on X[65536, 4096] fp32; 5 the 8-GPU scale-out problems (FA bf16 causal
# [64,32,8192,128], GEMM bf16 65536 x 16384 x 16384).
FA_F32 = FAConfig("fa_f32_B1_H4_S256_D64", 1, 4, 256, 64, False, torch.float32)
FA_F16_CAUSAL = FAConfig("fa_f16_causal_B4_H16_S2048_D128", 4, 16, 2048, 128, True,
                         torch.float16, 0.5)
FA_F16_CAUSAL_D64 = FAConfig("fa_f16_causal_B4_H16_S2048_D64", 4, 16, 2048, 64, True,
                             torch.float16, 0.5)
FA_F16_CAUSAL_D32 = FAConfig("fa_f16_causal_B4_H16_S2048_D32", 4, 16, 2048, 32, True,
                             torch.float16, 0.5)
FA_BF16_CAUSAL = FAConfig("fa_bf16_causal_B4_H16_S2048_D128", 4, 16, 2048, 128, True,
                          torch.bfloat16, 0.5)
FA_BF16_SCALE = FAConfig("fa_bf16_causal_B64_H32_S8192_D128", 64, 32, 8192, 128, True,
                         torch.bfloat16, 0.5)
GEMM_F16 = GemmConfig("gemm_f16_8192_bias_relu", 8192, 8192, 8192, torch.float16, True, "relu",
                      torch.float16)
GEMM_F32 = GemmConfig("gemm_f32_2048", 2048, 2048, 2048, torch.float32, False, "none",
                      torch.float32)
GEMM_BF16_SCALE = GemmConfig("gemm_bf16_65536x16384x16384", 65536, 16384, 16384, torch.bfloat16,
                             False, "none", torch.bfloat16)
ROWS_F32 = RowConfig("rows_f32_65536x4096", 65536, 4096, torch.float32)


def fa_inputs(cfg: FAConfig, device="cpu", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (cfg.B, cfg.H, cfg.S, cfg.D)
    out = []
    for _ in range(3):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        if cfg.std != 1.0:
            t.mul_(cfg.std)
        out.append(t.to(cfg.dtype))
    return out


def gemm_inputs(cfg: GemmConfig, device="cpu", seed: int = 0):
    """A, B ~ N(0,1)/sqrt(K); bias ~ N(0, 0.1) (fp32 bias, like the accumulator)."""
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(cfg.K)
    a = (torch.randn(cfg.M, cfg.K, generator=g, device=device) * s).to(cfg.dtype)
    b = (torch.randn(cfg.K, cfg.N, generator=g, device=device) * s).to(cfg.dtype)
    bias = (torch.randn(cfg.N, generator=g, device=device) * 0.1) if cfg.bias else None
    return a, b, bias


def row_inputs(cfg: RowConfig, device="cpu", seed: int = 0):
    """X ~ N(0,1); gamma ~ N(1, 0.1); beta ~ N(0, 0.1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(cfg.rows, cfg.cols, generator=g, device=device).to(cfg.dtype)
    w = (1.0 + 0.1 * torch.randn(cfg.cols, generator=g, device=device)).to(cfg.dtype)
    b = (0.1 * torch.randn(cfg.cols, generator=g, device=device)).to(cfg.dtype)
    return x, w, b
