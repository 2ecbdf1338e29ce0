"""torch.compile(backend="b2msl") over the reference's model list.

The reference compiles 33 small modules with torch.compile and compares each
with eager execution (tests/test_torch_compile.py:60-280: elementwise
activations, layer types, composite models up to a 4-layer GPT). The same
list runs here through the FX rewrite of this package:

* CPU (no GPU needed): Dynamo captures each module under ``torch.no_grad()``
  and the rewrite (``allow_cpu=True``, nothing executed) must replace exactly
  the hot-path patterns listed for it -- attention, linear/matmul (+ fused
  activation), softmax, LayerNorm, last-dim reductions -- and nothing else.
* GPU: the compiled module runs on CUDA, the same rewrites must fire, and its
  output is checked against the module evaluated in float64 on the CPU:
  max-abs <= 1e-4 * max(1, max|ref|) for float32 modules, normwise <= 2e-3
  for the float16 / bfloat16 ones (bf16 outputs get the 2^-8 storage
  allowance), exact argmax where the inputs have no ties.
"""
from __future__ import annotations

import copy

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import triton_msl_b200  # noqa: F401  (registers the backend)
from triton_msl_b200 import compile_backend as cb


# ------------------------------------------------------------------ modules
class _Fn(nn.Module):
    def __init__(self, fn):
        super().__init__()
        self.fn = fn

    def forward(self, x):
        return self.fn(x)


class _ResBlock(nn.Module):
    def __init__(self, ch=16):
        super().__init__()
        self.c1, self.b1 = nn.Conv2d(ch, ch, 3, padding=1), nn.BatchNorm2d(ch)
        self.c2, self.b2 = nn.Conv2d(ch, ch, 3, padding=1), nn.BatchNorm2d(ch)

    def forward(self, x):
        y = torch.relu(self.b1(self.c1(x)))
        return torch.relu(self.b2(self.c2(y)) + x)


class _DepthwiseSeparable(nn.Module):
    def __init__(self):
        super().__init__()
        self.dw = nn.Conv2d(32, 32, 3, padding=1, groups=32)
        self.pw = nn.Conv2d(32, 64, 1)
        self.bn = nn.BatchNorm2d(64)

    def forward(self, x):
        return torch.relu(self.bn(self.pw(self.dw(x))))


class _ConvNet(nn.Module):
    def __init__(self):
        super().__init__()
        self.features = nn.Sequential(
            nn.Conv2d(3, 32, 3, padding=1), nn.BatchNorm2d(32), nn.ReLU(),
            nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64), nn.ReLU(),
            nn.AdaptiveAvgPool2d(1))
        self.classifier = nn.Linear(64, 10)

    def forward(self, x):
        return self.classifier(self.features(x).flatten(1))


def _encoder_layer(d, heads, ff):
    return nn.TransformerEncoderLayer(d, heads, dim_feedforward=ff, batch_first=True, dropout=0.0)


class _MHA(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = nn.MultiheadAttention(128, 4, batch_first=True, dropout=0.0)

    def forward(self, x):
        return self.attn(x, x, x, need_weights=False)[0]


class _SmallGPT(nn.Module):
    def __init__(self):
        super().__init__()
        self.embedding = nn.Embedding(1000, 128)
        self.transformer = nn.TransformerEncoder(_encoder_layer(128, 4, 256), 2,
                                                 enable_nested_tensor=False)
        self.fc = nn.Linear(128, 1000)

    def forward(self, x):
        return self.fc(self.transformer(self.embedding(x)))


class _GPT4(nn.Module):
    def __init__(self):
        super().__init__()
        self.emb, self.pos = nn.Embedding(5000, 256), nn.Embedding(128, 256)
        self.transformer = nn.TransformerEncoder(_encoder_layer(256, 8, 512), 4,
                                                 enable_nested_tensor=False)
        self.head = nn.Linear(256, 5000)

    def forward(self, x):
        pos = torch.arange(x.size(1), device=x.device)[None]
        return self.head(self.transformer(self.emb(x) + self.pos(pos)))


class _MiniViT(nn.Module):
    def __init__(self, patch=4, d=128):
        super().__init__()
        self.patch_embed = nn.Conv2d(3, d, patch, stride=patch)
        self.cls_token = nn.Parameter(torch.randn(1, 1, d))
        self.encoder = nn.TransformerEncoder(_encoder_layer(d, 4, 256), 2, enable_nested_tensor=False)
        self.head = nn.Linear(d, 10)

    def forward(self, x):
        x = self.patch_embed(x).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(x.size(0), -1, -1), x], dim=1)
        return self.head(self.encoder(x)[:, 0])


class _LSTM(nn.Module):
    def __init__(self):
        super().__init__()
        self.lstm = nn.LSTM(64, 128, num_layers=2, batch_first=True)
        self.fc = nn.Linear(128, 10)

    def forward(self, x):
        return self.fc(self.lstm(x)[0][:, -1])


class _EmbBagMean(nn.Module):
    def __init__(self):
        super().__init__()
        self.emb = nn.Embedding(10000, 256)
        self.fc = nn.Linear(256, 64)

    def forward(self, x):
        return self.fc(self.emb(x).mean(dim=1))


class _CausalBlock(nn.Module):
    """Pre-norm decoder block written with the functional calls models use."""

    def __init__(self, d=256, h=4):
        super().__init__()
        self.h = h
        self.ln1, self.ln2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.qkv, self.proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
        self.up, self.down = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)

    def forward(self, x):
        B, S, D = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(B, S, 3, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(a.transpose(1, 2).reshape(B, S, D))
        return x + self.down(F.gelu(self.up(self.ln2(x))))


class _Head(nn.Module):
    """Classifier head: RMSNorm, logits, softmax, argmax and a row sum."""

    def __init__(self, d=512, n=128):
        super().__init__()
        self.w = nn.Parameter(torch.rand(d) + 0.5)
        self.fc = nn.Linear(d, n)

    def forward(self, x):
        y = self.fc(F.rms_norm(x, (x.shape[-1],), self.w, 1e-6))
        return torch.softmax(y, dim=-1), y.argmax(dim=-1), y.sum(-1)


def _softmax(x):
    return torch.softmax(x, dim=-1)


def _log_softmax(x):
    return torch.log_softmax(x, dim=-1)


def _randn(*shape):
    def make():
        return torch.randn(*shape, generator=torch.Generator().manual_seed(7))
    return make


def _randint(hi, *shape):
    def make():
        return torch.randint(0, hi, shape, generator=torch.Generator().manual_seed(7))
    return make


# Each case: (name, module factory, input factory, rewrite tags expected, dtype).
# nn.TransformerEncoderLayer in inference reaches the graph as its fused
# fast-path op (torch._transformer_encoder_layer_fwd) and nn.MultiheadAttention
# as F.multi_head_attention_forward (or the native fused op): both are
# rewritten whole ("encoder_layer", "attention(mha)") into the projection
# GEMMs, the attention kernel and the LayerNorms. Dynamo does not capture
# nn.LSTM's frame, so that model runs as eager code and nothing is rewritten.
_TLAYER = ["encoder_layer"]
CASES = [
    # elementwise (reference TestElementwise): nothing on the hot path
    ("identity", lambda: nn.Identity(), _randn(1024), [], torch.float32),
    ("relu", lambda: nn.ReLU(), _randn(1024), [], torch.float32),
    ("gelu", lambda: nn.GELU(), _randn(1024), [], torch.float32),
    ("silu", lambda: nn.SiLU(), _randn(1024), [], torch.float32),
    ("sigmoid", lambda: nn.Sigmoid(), _randn(1024), [], torch.float32),
    ("tanh", lambda: nn.Tanh(), _randn(1024), [], torch.float32),
    ("elu", lambda: nn.ELU(), _randn(1024), [], torch.float32),
    ("leaky_relu", lambda: nn.LeakyReLU(0.2), _randn(1024), [], torch.float32),
    ("dropout_in_eval", lambda: nn.Dropout(0.5), _randn(1024), [], torch.float32),
    # layer types (reference TestLayers)
    ("linear", lambda: nn.Linear(128, 64), _randn(32, 128), ["linear"], torch.float32),
    ("layer_norm", lambda: nn.LayerNorm(128), _randn(32, 128), ["layer_norm"], torch.float32),
    ("batch_norm_2d", lambda: nn.BatchNorm2d(16), _randn(2, 16, 8, 8), [], torch.float32),
    ("group_norm", lambda: nn.GroupNorm(4, 16), _randn(2, 16, 8, 8), [], torch.float32),
    ("instance_norm", lambda: nn.InstanceNorm2d(16, affine=True), _randn(2, 16, 8, 8), [], torch.float32),
    ("embedding", lambda: nn.Embedding(1000, 128), _randint(1000, 2, 16), [], torch.float32),
    ("conv2d", lambda: nn.Conv2d(3, 16, 3, padding=1), _randn(1, 3, 32, 32), [], torch.float32),
    ("avg_pool", lambda: nn.AvgPool2d(2), _randn(1, 16, 8, 8), [], torch.float32),
    ("max_pool", lambda: nn.MaxPool2d(2), _randn(1, 16, 8, 8), [], torch.float32),
    ("softmax", lambda: _Fn(_softmax), _randn(32, 128), ["softmax"], torch.float32),
    ("log_softmax", lambda: _Fn(_log_softmax), _randn(32, 128), [], torch.float32),
    # composite models (reference TestModels)
    ("mlp", lambda: nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 64)),
     _randn(32, 128), ["linear+relu", "linear"], torch.float32),
    ("large_mlp", lambda: nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 512), nn.GELU(),
                                        nn.Linear(512, 256)),
     _randn(16, 256), ["linear+gelu", "linear+gelu", "linear"], torch.float32),
    ("res_block", _ResBlock, _randn(1, 16, 8, 8), [], torch.float32),
    ("depthwise_separable", _DepthwiseSeparable, _randn(2, 32, 8, 8), [], torch.float32),
    ("convnet", _ConvNet, _randn(4, 3, 16, 16), ["linear"], torch.float32),
    ("transformer_block", lambda: _encoder_layer(128, 4, 256), _randn(2, 16, 128), _TLAYER, torch.float32),
    ("multihead_attention", _MHA, _randn(2, 16, 128), ["attention(mha)"], torch.float32),
    ("small_gpt", _SmallGPT, _randint(1000, 2, 16), _TLAYER * 2 + ["linear"], torch.float32),
    ("gpt_4layer", _GPT4, _randint(5000, 2, 32), _TLAYER * 4 + ["linear"], torch.float32),
    ("mini_vit", _MiniViT, _randn(2, 3, 16, 16), _TLAYER * 2 + ["linear"], torch.float32),
    ("lstm", _LSTM, _randn(4, 16, 64), [], torch.float32),
    ("embedding_bag_mean", _EmbBagMean, _randint(10000, 8, 32), ["linear"], torch.float32),
    # the hot path in half precision
    ("causal_block_f16", _CausalBlock, _randn(2, 128, 256),
     ["layer_norm", "linear", "attention", "linear", "layer_norm", "linear+gelu", "linear"], torch.float16),
    ("causal_block_bf16", _CausalBlock, _randn(2, 128, 256),
     ["layer_norm", "linear", "attention", "linear", "layer_norm", "linear+gelu", "linear"], torch.bfloat16),
    ("head_f32", _Head, _randn(64, 512), ["rms_norm", "linear", "softmax", "row_argmax", "row_sum"],
     torch.float32),
]
IDS = [c[0] for c in CASES]


@pytest.fixture(autouse=True)
def _exact_fp32_library_kernels():
    # the fp64 comparison wants float32 convolutions / RNNs / matmuls outside
    # the rewritten nodes in full fp32, not TF32
    old = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = old


def _prep(mk, inp, dtype, device):
    torch.manual_seed(0)
    m = mk().eval()
    x = inp()
    if x.is_floating_point():
        x = x.to(dtype)
    return m.to(device=device, dtype=dtype), x.to(device)


def _capture_tags(m, x):
    graphs = []

    def grab(gm, ex):
        graphs.append(gm)
        return gm.forward

    torch._dynamo.reset()
    with torch.no_grad():
        torch.compile(m, backend=grab)(x)
    tags = []
    for gm in graphs:
        tags += cb.rewrite(gm, allow_cpu=True)
    return tags


@pytest.mark.parametrize("name,mk,inp,expected,dtype", CASES, ids=IDS)
def test_rewrite_tags_cpu(name, mk, inp, expected, dtype):
    m, x = _prep(mk, inp, torch.float32, "cpu")
    assert sorted(_capture_tags(m, x)) == sorted(expected)


def _outputs(y):
    return list(y) if isinstance(y, (tuple, list)) else [y]


@pytest.mark.gpu
@pytest.mark.parametrize("name,mk,inp,expected,dtype", CASES, ids=IDS)
def test_compiled_matches_fp64_reference_gpu(name, mk, inp, expected, dtype):
    m, x = _prep(mk, inp, dtype, "cuda")
    ref_m = copy.deepcopy(m).to(device="cpu", dtype=torch.float64)
    xr = x.cpu().to(torch.float64) if x.is_floating_point() else x.cpu()
    with torch.no_grad():
        refs = _outputs(ref_m(xr))
    torch._dynamo.reset()
    cb.rewrite_log.clear()
    with torch.no_grad():
        got = _outputs(torch.compile(m, backend="b2msl")(x))
    assert sorted(cb.rewrite_log) == sorted(expected)
    for g, r in zip(got, refs):
        if g.dtype == torch.int64:
            assert torch.equal(g.cpu(), r), "argmax differs"
            continue
        g = g.double().cpu()
        scale = max(1.0, r.abs().max().item())
        err = (g - r).abs().max().item()
        if dtype == torch.float32:
            assert err <= 1e-4 * scale, f"max-abs {err:.3e} > {1e-4 * scale:.3e}"
        else:
            tol = 2e-3 + (2.0 ** -8 if dtype == torch.bfloat16 else 0.0)
            rel = err / max(r.abs().max().item(), 1e-6)
            assert rel <= tol, f"normwise {rel:.3e} > {tol:.3e}"
