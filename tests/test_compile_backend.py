"""torch.compile backend: the FX rewrite recognises the hot-path patterns the
reference's detectors handle (attention, matmul + epilogue, softmax /
LayerNorm / RMSNorm, last-dim reductions). CPU tests capture the Dynamo graph
and check the rewrite (allow_cpu=True, nothing executed); the GPU test runs the
compiled module and compares with eager (reference test_torch_compile.py:39-58
style: compiled vs eager)."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import triton_msl_b200  # noqa: F401  (registers the backend)
from triton_msl_b200 import compile_backend as cb


class Block(nn.Module):
    def __init__(self, d=64, h=4):
        super().__init__()
        self.h = h
        self.ln = nn.LayerNorm(d)
        self.qkv = nn.Linear(d, 3 * d)
        self.up = nn.Linear(d, 4 * d)
        self.down = nn.Linear(4 * d, d)

    def forward(self, x):
        B, S, D = x.shape
        y = self.ln(x)
        q, k, v = self.qkv(y).view(B, S, 3, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + a.transpose(1, 2).reshape(B, S, D)
        x = x + self.down(F.relu(self.up(x)))
        return torch.softmax(x, dim=-1), x.argmax(dim=-1), x.sum(-1)


class ExplicitAttn(nn.Module):
    def forward(self, q, k, v):
        return torch.softmax(q @ k.transpose(-2, -1) * 0.125, dim=-1) @ v


class Norms(nn.Module):
    def __init__(self, d=96):
        super().__init__()
        self.w = nn.Parameter(torch.ones(d))

    def forward(self, x, a, b):
        return F.rms_norm(x, (x.shape[-1],), self.w, 1e-6), torch.amax(x, -1), F.gelu(a @ b)


def _capture(mod, *inputs):
    graphs = []

    def grab(gm, ex):
        graphs.append(gm)
        return gm.forward

    torch._dynamo.reset()
    with torch.no_grad():
        torch.compile(mod, backend=grab, fullgraph=False)(*inputs)
    return graphs


def _rewrite_all(mod, *inputs):
    tags = []
    for gm in _capture(mod, *inputs):
        tags += cb.rewrite(gm, allow_cpu=True)
    return tags


def test_rewrites_transformer_block_patterns():
    tags = _rewrite_all(Block(), torch.randn(2, 16, 64))
    assert "layer_norm" in tags
    assert "attention" in tags
    assert "linear" in tags and "linear+relu" in tags
    assert "softmax" in tags and "row_argmax" in tags and "row_sum" in tags


def test_rewrites_explicit_attention_chain():
    q = torch.randn(1, 2, 32, 16)
    assert "attention(explicit)" in _rewrite_all(ExplicitAttn(), q, q, q)


def test_rewrites_norms_and_matmul_epilogue():
    tags = _rewrite_all(Norms(), torch.randn(8, 96), torch.randn(16, 32), torch.randn(32, 24))
    assert "rms_norm" in tags and "row_max" in tags and "matmul+gelu" in tags


def test_cpu_tensors_are_left_alone_by_default():
    for gm in _capture(Block(), torch.randn(2, 16, 64)):
        assert cb.rewrite(gm) == []


def test_backend_registered():
    from torch._dynamo.backends.registry import list_backends
    assert "b2msl" in list_backends()


def test_training_graph_is_left_to_autograd():
    """The ops are forward-only: with parameters that require grad and grad
    mode on, nothing differentiable is rewritten (an argmax has no gradient and
    still may be), so backward is PyTorch's own."""
    graphs = []

    def grab(gm, ex):
        graphs.append(gm)
        return gm.forward

    torch._dynamo.reset()
    torch.compile(Block(), backend=grab)(torch.randn(2, 16, 64))
    assert graphs
    for gm in graphs:
        assert cb.rewrite(gm, allow_cpu=True) == ["row_argmax"]


@pytest.mark.gpu
def test_compiled_block_matches_eager_on_gpu():
    torch.manual_seed(0)
    m = Block(d=128, h=2).cuda().half().eval()
    x = torch.randn(2, 256, 128, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        ref = Block(d=128, h=2).double()
        ref.load_state_dict({k: v.double().cpu() for k, v in m.state_dict().items()})
        refs = ref(x.double().cpu())
        torch._dynamo.reset()
        cb.rewrite_log.clear()
        got = torch.compile(m, backend="b2msl")(x)
    assert sorted(cb.rewrite_log) == sorted(["layer_norm", "linear", "attention", "linear+relu",
                                             "linear", "softmax", "row_argmax", "row_sum"])
    soft, idx, tot = got
    rsoft, ridx, rtot = refs
    for g, r in ((soft, rsoft), (tot, rtot)):
        err = (g.double().cpu() - r).abs().max().item() / max(r.abs().max().item(), 1e-6)
        assert err <= 2e-3, err
    # argmax of the fp16 residual stream: exact wherever the top two fp64
    # values are further apart than the fp16 error of the row
    x_ref = torch.log(rsoft)  # softmax is monotone: same ordering as the logits
    v2 = x_ref.topk(2, dim=-1).values
    clear = (v2[..., 0] - v2[..., 1]) > 2e-2
    assert clear.float().mean() > 0.5
    assert torch.equal(idx.cpu()[clear], ridx[clear])


@pytest.mark.gpu
def test_compiled_training_step_keeps_gradients():
    torch.manual_seed(0)
    m = Block(d=128, h=2).cuda()
    x = torch.randn(2, 64, 128, device="cuda")
    ref = Block(d=128, h=2).cuda()
    ref.load_state_dict(m.state_dict())
    torch._dynamo.reset()
    cb.rewrite_log.clear()
    out = torch.compile(m, backend="b2msl")(x)[0].sum()
    out.backward()
    ref(x)[0].sum().backward()
    assert cb.rewrite_log == ["row_argmax"]
    for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
        assert torch.allclose(p.grad, q.grad, atol=1e-5, rtol=1e-4), n


class MatmulSoftmax(nn.Module):
    def forward(self, a, b):
        return torch.softmax(a @ b, dim=-1)


def test_rewrites_matmul_softmax_into_gemm_epilogue():
    tags = _rewrite_all(MatmulSoftmax(), torch.randn(64, 32), torch.randn(32, 128))
    assert "matmul+softmax" in tags
    tags = _rewrite_all(MatmulSoftmax(), torch.randn(64, 32), torch.randn(32, 512))
    assert "matmul+softmax" not in tags    # N > 256: separate softmax


class LinearChain(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc = nn.Linear(64, 96)

    def forward(self, x, a, b):
        y = torch.clamp(self.fc(x) * 0.5 - 0.1, min=-1.0, max=2.0).exp()
        z = torch.sigmoid(1.0 - (a @ b) / 3.0)
        return y, z, torch.relu(a @ b)


def test_rewrites_general_epilogue_chains():
    tags = _rewrite_all(LinearChain(), torch.randn(8, 64), torch.randn(16, 32), torch.randn(32, 24))
    # bias, mul, sub, clamp, exp  /  div, rsub, sigmoid  /  a single ReLU stays an activation
    assert sorted(tags) == sorted(["linear+chain5", "matmul+chain3", "matmul+relu"])


@pytest.mark.gpu
def test_compiled_epilogue_chains_match_fp64_on_gpu():
    torch.manual_seed(0)
    m = LinearChain().cuda().half().eval()
    x = torch.randn(256, 64, device="cuda", dtype=torch.float16)
    a = torch.randn(256, 128, device="cuda", dtype=torch.float16) / 8
    b = torch.randn(128, 192, device="cuda", dtype=torch.float16) / 8
    ref_m = LinearChain().double()
    ref_m.load_state_dict({k: v.double().cpu() for k, v in m.state_dict().items()})
    with torch.no_grad():
        refs = ref_m(x.double().cpu(), a.double().cpu(), b.double().cpu())
        torch._dynamo.reset()
        cb.rewrite_log.clear()
        got = torch.compile(m, backend="b2msl")(x, a, b)
    assert sorted(cb.rewrite_log) == sorted(["linear+chain5", "matmul+chain3", "matmul+relu"])
    for g, r in zip(got, refs):
        err = (g.double().cpu() - r).abs().max().item() / max(r.abs().max().item(), 1e-6)
        assert err <= 2e-3, err


class AxisReductions(nn.Module):
    def forward(self, x, y):
        return x.sum(0), torch.amax(y, dim=1), y.argmin(dim=0), x.sum(-1)


def test_rewrites_reductions_along_any_axis():
    tags = _rewrite_all(AxisReductions(), torch.randn(64, 96), torch.randn(8, 16, 32))
    assert sorted(tags) == sorted(["reduce_sum(dim)", "reduce_max(dim)", "reduce_argmin(dim)", "row_sum"])
