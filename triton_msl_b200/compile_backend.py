"""``torch.compile`` backend that routes the hot-path patterns to the b2msl ops.

The reference reaches its templates from ``torch.compile`` by registering a
Triton scheduling for MPS (``register_metal_triton_backend``,
triton_msl/inductor/__init__.py:52-153) and letting its pattern detectors
(attention ``generic_lowerer.py:679-835``, matmul epilogue
``_lowerer_detection.py:1150-1364``, softmax / LayerNorm
``_lowerer_detection.py:1828-2074``) pick templates from the generated
kernels. Here the same patterns are recognised directly in the FX graph that
Dynamo captures and replaced by calls to the custom ops:

* ``F.scaled_dot_product_attention(q, k, v[, is_causal, scale])`` and the
  explicit ``softmax(q @ k.transpose(-2, -1) * s) @ v`` chain -> ``flash_attn_fwd``
* ``F.linear(x, w[, b])`` / ``torch.matmul`` / ``@`` / ``torch.addmm`` on 2-D
  operands, with a following ``relu`` / ``gelu`` / ``silu`` or a last-dim
  ``softmax`` (N <= 256, the fused matmul-softmax) folded in -> ``gemm``
* ``softmax(x, dim=-1)``, ``F.layer_norm`` over the last dim, ``F.rms_norm``
  over the last dim, ``sum / amax / amin / argmax / argmin(dim=-1)`` -> row ops

A node is rewritten only when its traced example value says the replacement
is exact: CUDA tensors, float32/float16/bfloat16, shapes the ops accept, and
no autograd history needed. The ops are forward-only (the reference's
templates are forward kernels too), so a node whose output requires grad --
a training graph -- is left to PyTorch and backward stays correct; compile
under ``torch.no_grad()`` / ``torch.inference_mode()`` (or with parameters
that do not require grad) to route the patterns. The rest of the graph runs
as captured (``inner="eager"``) or through Inductor
(``inner="inductor"``).
"""
from __future__ import annotations

import operator
from typing import Callable, List, Optional

import torch
import torch.fx as fx
import torch.nn.functional as F

from . import ops as b2ops

_FLOATS = (torch.float32, torch.float16, torch.bfloat16)
_EPI_MAX = 16


def _val(n):
    if isinstance(n, fx.Node):
        return n.meta.get("example_value", n.meta.get("val"))
    return None


def _ok_tensor(n, allow_cpu: bool, ndim: Optional[int] = None) -> bool:
    v = _val(n)
    if not isinstance(v, torch.Tensor):
        return False
    if v.dtype not in _FLOATS:
        return False
    if not allow_cpu and v.device.type != "cuda":
        return False
    if ndim is not None and v.dim() != ndim:
        return False
    return True


def _arg(node: fx.Node, i: int, name: str, default=None):
    if len(node.args) > i:
        return node.args[i]
    return node.kwargs.get(name, default)


def _is_last_dim(dim, v) -> bool:
    if isinstance(dim, (list, tuple)):
        if len(dim) != 1:
            return False
        dim = dim[0]
    return isinstance(dim, int) and v is not None and dim in (-1, v.dim() - 1)


_SOFTMAX = {torch.softmax, F.softmax, torch.nn.functional.softmax, "softmax"}
_MATMUL = {torch.matmul, operator.matmul, torch.mm, "matmul", "mm"}
_ACTS = {torch.relu: "relu", F.relu: "relu", "relu": "relu", F.gelu: "gelu",
         F.silu: "silu", torch.nn.functional.silu: "silu"}
_LINEAR = {F.linear, torch._C._nn.linear}
_LAYERNORM = {F.layer_norm, torch.layer_norm}
_RMSNORM = {f for f in (getattr(F, "rms_norm", None), getattr(torch, "rms_norm", None)) if f is not None}
_ROWRED = {torch.sum: "sum", "sum": "sum", torch.amax: "max", "amax": "max",
           torch.amin: "min", "amin": "min", torch.argmax: "argmax", "argmax": "argmax",
           torch.argmin: "argmin", "argmin": "argmin"}


def _target_key(node: fx.Node):
    if node.op == "call_method":
        return node.target
    if node.op == "call_function":
        return node.target
    return None


def _in(node, table) -> bool:
    k = _target_key(node)
    try:
        return k in table
    except TypeError:
        return False


# ------------------------------------------------------------ replacements
def _linear_act(x, w, b, act):
    """x[..., K] @ w[N, K]^T (+ b) with activation, through the GEMM op."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    y = b2ops.gemm(x2, w.t(), b, act)
    return y.reshape(*lead, w.shape[0])


def _matmul_act(a, b, act):
    return b2ops.gemm(a, b, None, act)


def _addmm_act(bias, a, b, act):
    return b2ops.gemm(a, b, bias, act)


def _linear_chain(x, w, b, codes, args):
    """x[..., K] @ w[N, K]^T with a general epilogue chain (bias first when given)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.ops.b2msl.gemm_epilogue(x2, w.t(), b, list(codes), list(args), None)
    return y.reshape(*lead, w.shape[0])


def _matmul_chain(a, b, bias, codes, args):
    return torch.ops.b2msl.gemm_epilogue(a, b, bias, list(codes), list(args), None)


def _num(x) -> bool:
    return isinstance(x, (int, float)) and not isinstance(x, bool)


_UNARY_EPI = {torch.exp: "exp", torch.exp2: "exp2", torch.log: "log", torch.log2: "log2",
              torch.sqrt: "sqrt", torch.rsqrt: "rsqrt", torch.sin: "sin", torch.cos: "cos",
              torch.erf: "erf", torch.special.erf: "erf", torch.tanh: "tanh", torch.floor: "floor",
              torch.ceil: "ceil", torch.abs: "abs", torch.sigmoid: "sigmoid", F.sigmoid: "sigmoid",
              torch.neg: "neg", operator.neg: "neg", torch.relu: "relu", F.relu: "relu",
              F.silu: "silu", "exp": "exp", "exp2": "exp2", "log": "log", "log2": "log2",
              "sqrt": "sqrt", "rsqrt": "rsqrt", "sin": "sin", "cos": "cos", "erf": "erf",
              "tanh": "tanh", "floor": "floor", "ceil": "ceil", "abs": "abs",
              "sigmoid": "sigmoid", "neg": "neg", "relu": "relu"}


def _epi_step(u: fx.Node, prev: fx.Node):
    """The epilogue op(s) element-wise node u applies to its input prev, or None.
    Constants must be Python numbers (the traced graph's literals)."""
    if u.op not in ("call_function", "call_method"):
        return None
    t = _target_key(u)
    kw = {k: v for k, v in u.kwargs.items() if not (k == "inplace" and v is False)}
    a = u.args
    try:
        if t in _UNARY_EPI and len(a) == 1 and a[0] is prev and not kw:
            return [(_UNARY_EPI[t],)]
    except TypeError:
        return None
    if t is F.gelu and len(a) == 1 and a[0] is prev and kw.get("approximate", "none") in ("none", "tanh") \
            and set(kw) <= {"approximate"}:
        return [("gelu_tanh",) if kw.get("approximate") == "tanh" else ("gelu",)]
    if kw:
        if t in (torch.clamp, "clamp", torch.clip, "clip") and len(a) == 1 and a[0] is prev \
                and set(kw) <= {"min", "max"}:
            lo, hi = kw.get("min"), kw.get("max")
            if (lo is None or _num(lo)) and (hi is None or _num(hi)):
                return [("clamp", float("-inf") if lo is None else lo, float("inf") if hi is None else hi)]
        return None
    if t in (torch.clamp, "clamp", torch.clip, "clip") and 2 <= len(a) <= 3 and a[0] is prev:
        lo = a[1]
        hi = a[2] if len(a) == 3 else None
        if (lo is None or _num(lo)) and (hi is None or _num(hi)):
            return [("clamp", float("-inf") if lo is None else lo, float("inf") if hi is None else hi)]
        return None
    if len(a) != 2:
        return None
    x, y = a
    if t in (operator.add, torch.add, "add", operator.iadd):
        if x is prev and _num(y):
            return [("add", y)]
        if y is prev and _num(x):
            return [("add", x)]
    if t in (operator.sub, torch.sub, "sub", operator.isub):
        if x is prev and _num(y):
            return [("sub", y)]
        if y is prev and _num(x):
            return [("rsub", x)]
    if t in (operator.mul, torch.mul, "mul", operator.imul):
        if x is prev and _num(y):
            return [("mul", y)]
        if y is prev and _num(x):
            return [("mul", x)]
    if t in (operator.truediv, torch.div, "div", torch.true_divide, "true_divide"):
        if x is prev and _num(y):
            return [("div", y)]
        if y is prev and _num(x):
            return [("rdiv", x)]
    return None


def _sdpa(q, k, v, causal, scale):
    return b2ops.flash_attn_fwd(q, k, v, causal=causal, sm_scale=scale)


def _mha_core(x_q, x_k, x_v, num_heads, w_in, b_in, w_out, b_out, causal, batch_first):
    """Multi-head attention with packed input projection through the b2msl ops:
    in-projection GEMMs, the heads as strided [B, H, S, Dh] views into the
    projection output (the attention kernel takes any strides), attention,
    out-projection GEMM. Inputs are [B, S, E] when batch_first else [S, B, E]."""
    if not batch_first:
        x_q, x_k, x_v = (t.transpose(0, 1) for t in (x_q, x_k, x_v))
    B, S, E = x_q.shape
    Dh = E // num_heads
    if x_q is x_k and x_k is x_v:
        qkv = _linear_act(x_q, w_in, b_in, "none").view(B, S, 3, num_heads, Dh)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
    else:
        ws = w_in.chunk(3)
        bs = b_in.chunk(3) if b_in is not None else (None, None, None)
        q, k, v = (_linear_act(t, w_, b_, "none").view(B, t.shape[1], num_heads, Dh).transpose(1, 2)
                   for t, w_, b_ in zip((x_q, x_k, x_v), ws, bs))
    o = b2ops.flash_attn_fwd(q, k, v, causal=causal, sm_scale=Dh ** -0.5)
    o = o.transpose(1, 2).reshape(B, S, E)
    y = _linear_act(o, w_out, b_out, "none")
    return y if batch_first else y.transpose(0, 1)


def _mha_functional(q, k, v, num_heads, w_in, b_in, w_out, b_out, causal):
    """F.multi_head_attention_forward (sequence-first inputs) -> (out, None)."""
    return _mha_core(q, k, v, num_heads, w_in, b_in, w_out, b_out, causal, False), None


def _mha_native(q, k, v, num_heads, w_in, b_in, w_out, b_out):
    """torch._native_multi_head_attention (batch-first inputs) -> (out, None)."""
    return _mha_core(q, k, v, num_heads, w_in, b_in, w_out, b_out, False, True), None


def _encoder_layer(x, num_heads, w_in, b_in, w_out, b_out, use_gelu, norm_first, eps,
                   n1w, n1b, n2w, n2b, l1w, l1b, l2w, l2b):
    """The inference fast path of nn.TransformerEncoderLayer
    (torch._transformer_encoder_layer_fwd, batch-first, no mask) through the
    b2msl ops: self-attention, LayerNorms and the feed-forward GEMMs with the
    activation fused into the first."""
    act = "gelu" if use_gelu else "relu"

    def ff(t):
        return _linear_act(_linear_act(t, l1w, l1b, act), l2w, l2b, "none")

    def sa(t):
        return _mha_core(t, t, t, num_heads, w_in, b_in, w_out, b_out, False, True)

    if norm_first:
        x = x + sa(b2ops.row_layernorm(x, n1w, n1b, eps))
        return x + ff(b2ops.row_layernorm(x, n2w, n2b, eps))
    x = b2ops.row_layernorm(x + sa(x), n1w, n1b, eps)
    return b2ops.row_layernorm(x + ff(x), n2w, n2b, eps)


def _rowred(x, kind):
    return getattr(b2ops, f"row_{kind}")(x)


def _axisred(x, kind, dim):
    return b2ops.reduce(x, kind, dim)


def _layer_norm(x, w, b, eps):
    return b2ops.row_layernorm(x, w, b, eps)


def _rms_norm(x, w, eps):
    return b2ops.row_rmsnorm(x, w, eps)


class Rewriter:
    """Pattern-rewrites one FX graph in place; counts what it replaced."""

    def __init__(self, gm: fx.GraphModule, allow_cpu: bool = False):
        self.gm = gm
        self.g = gm.graph
        self.allow_cpu = allow_cpu
        self.replaced: List[str] = []

    def _replace(self, node: fx.Node, fn: Callable, args, tag: str, last: Optional[fx.Node] = None):
        anchor = last or node
        with self.g.inserting_after(anchor):
            new = self.g.call_function(fn, tuple(args))
        new.meta.update(anchor.meta)
        anchor.replace_all_uses_with(new)
        self.replaced.append(tag)
        return new

    def _epilogue_chain(self, node: fx.Node, has_bias: bool):
        """The longest run of single-user element-wise nodes after `node` that the
        general GEMM epilogue expresses (reference op chain, _lowerer_templates.py:
        1733-1855). Returns (last node, ops) when it is more than one activation."""
        ops = [("add_bias",)] if has_bias else []
        prev, last = node, None
        while len(prev.users) == 1 and len(ops) < _EPI_MAX:
            u = next(iter(prev.users))
            step = _epi_step(u, prev)
            v = _val(u)
            if step is None or not isinstance(v, torch.Tensor) or v.dtype != _val(node).dtype:
                break
            ops += step
            prev = last = u
        body = ops[1:] if has_bias else ops
        if last is None or (len(body) == 1 and body[0][0] in ("relu", "gelu", "gelu_tanh", "silu")):
            return None, None
        return last, ops

    def _single_user_act(self, node: fx.Node):
        users = list(node.users)
        if len(users) != 1:
            return None, None
        u = users[0]
        kw = {k: v for k, v in u.kwargs.items() if not (k == "inplace" and v is False)}
        if u.op in ("call_function", "call_method") and _in(u, _ACTS) and len(u.args) == 1 and \
                (not kw or (u.target is F.gelu and kw == {"approximate": "none"})):
            return u, _ACTS[_target_key(u)]
        if u.op == "call_function" and u.target is F.gelu and kw == {"approximate": "tanh"}:
            return u, "gelu_tanh"
        # matmul -> row softmax (the reference's fused matmul-softmax template),
        # when one output tile covers a row
        if _in(u, _SOFTMAX) and u.args and u.args[0] is node and u.kwargs.get("dtype") is None:
            v = _val(node)
            if v is not None and _is_last_dim(_arg(u, 1, "dim"), v) and v.shape[-1] <= 256:
                return u, "softmax"
        return None, None

    def _fusable_producer(self, x: fx.Node) -> bool:
        """x is a 2-D matmul / linear / addmm this pass will rewrite to a GEMM whose
        output rows fit one tile (N <= 256)."""
        v = _val(x)
        if v is None or v.shape[-1] > 256:
            return False
        ac = self.allow_cpu
        if _in(x, _MATMUL) and len(x.args) == 2:
            return _ok_tensor(x.args[0], ac, 2) and _ok_tensor(x.args[1], ac, 2)
        if _in(x, _LINEAR):
            return _ok_tensor(x.args[0], ac) and _ok_tensor(x.args[1], ac, 2)
        if _target_key(x) is torch.addmm and len(x.args) == 3:
            return all(_ok_tensor(a, ac) for a in x.args)
        return False

    def run(self) -> List[str]:
        # Consumers first, so a chain (softmax inside explicit attention, an
        # activation after a matmul) is seen whole before its parts.
        for node in reversed(list(self.g.nodes)):
            if node.op not in ("call_function", "call_method") or not node.users:
                continue
            try:
                self._visit(node)
            except Exception:  # a pattern that does not fit leaves the node alone
                continue
        self.g.eliminate_dead_code()
        self.gm.recompile()
        return self.replaced

    def _visit(self, node: fx.Node):
        out = _val(node)
        if isinstance(out, torch.Tensor) and out.requires_grad:
            return  # forward-only ops: keep autograd's own graph for training
        t = _target_key(node)
        ac = self.allow_cpu
        # ---- attention
        if t is F.scaled_dot_product_attention:
            q, k, v = node.args[:3]
            mask = _arg(node, 3, "attn_mask")
            drop = _arg(node, 4, "dropout_p", 0.0)
            causal = _arg(node, 5, "is_causal", False)
            scale = node.kwargs.get("scale")
            if mask is None and drop == 0.0 and all(_ok_tensor(x, ac, 4) for x in (q, k, v)):
                qv, kv, vv = (_val(x) for x in (q, k, v))
                if qv.shape == kv.shape == vv.shape and qv.dtype == kv.dtype == vv.dtype \
                        and qv.shape[-1] <= 128:
                    s = scale if scale is not None else qv.shape[-1] ** -0.5
                    self._replace(node, _sdpa, (q, k, v, bool(causal), float(s)), "attention")
            return
        # ---- nn.MultiheadAttention / nn.TransformerEncoderLayer inference paths
        if t is F.multi_head_attention_forward:
            self._visit_mha_functional(node)
            return
        if t is getattr(torch, "_native_multi_head_attention", None):
            self._visit_mha_native(node)
            return
        if t is getattr(torch, "_transformer_encoder_layer_fwd", None):
            self._visit_encoder_layer(node)
            return
        # ---- explicit attention chain: matmul(softmax(matmul(q, k^T) * s), v)
        if _in(node, _MATMUL) and len(node.args) == 2:
            p, v = node.args
            if isinstance(p, fx.Node) and _in(p, _SOFTMAX) and len(p.users) == 1:
                hit = self._explicit_attention(node, p, v)
                if hit:
                    return
            a, b = node.args
            if _ok_tensor(a, ac, 2) and _ok_tensor(b, ac, 2) and _val(a).dtype == _val(b).dtype:
                last, ops = self._epilogue_chain(node, False)
                if last is not None:
                    codes, args = b2ops._epi_program(ops)
                    self._replace(node, _matmul_chain, (a, b, None, codes, args),
                                  f"matmul+chain{len(ops)}", last)
                    return
                act_node, act = self._single_user_act(node)
                self._replace(node, _matmul_act, (a, b, act or "none"),
                              "matmul" + (f"+{act}" if act else ""), act_node)
            return
        # ---- linear (+ activation)
        if _in(node, _LINEAR):
            x, w = node.args[:2]
            b = _arg(node, 2, "bias")
            if _ok_tensor(x, ac) and _ok_tensor(w, ac, 2) and _val(x).dtype == _val(w).dtype \
                    and (b is None or _ok_tensor(b, ac, 1)):
                last, ops = self._epilogue_chain(node, b is not None)
                if last is not None:
                    codes, args = b2ops._epi_program(ops)
                    self._replace(node, _linear_chain, (x, w, b, codes, args),
                                  f"linear+chain{len(ops)}", last)
                    return
                act_node, act = self._single_user_act(node)
                self._replace(node, _linear_act, (x, w, b, act or "none"),
                              "linear" + (f"+{act}" if act else ""), act_node)
            return
        if t is torch.addmm and len(node.args) == 3 and not node.kwargs:
            bias, a, b = node.args
            if _ok_tensor(bias, ac, 1) and _ok_tensor(a, ac, 2) and _ok_tensor(b, ac, 2):
                last, ops = self._epilogue_chain(node, True)
                if last is not None:
                    codes, args = b2ops._epi_program(ops)
                    self._replace(node, _matmul_chain, (a, b, bias, codes, args),
                                  f"addmm+chain{len(ops)}", last)
                    return
                act_node, act = self._single_user_act(node)
                self._replace(node, _addmm_act, (bias, a, b, act or "none"),
                              "addmm" + (f"+{act}" if act else ""), act_node)
            return
        # ---- row family
        if _in(node, _SOFTMAX):
            x = node.args[0]
            dim = _arg(node, 1, "dim")
            if isinstance(x, fx.Node) and len(x.users) == 1 and self._fusable_producer(x):
                return  # the producing matmul absorbs it as a softmax epilogue
            if _ok_tensor(x, ac) and _is_last_dim(dim, _val(x)) and node.kwargs.get("dtype") is None:
                self._replace(node, b2ops.row_softmax, (x,), "softmax")
            return
        if _in(node, _LAYERNORM):
            x, shape = node.args[:2]
            w = _arg(node, 2, "weight")
            b = _arg(node, 3, "bias")
            eps = _arg(node, 4, "eps", 1e-5)
            xv = _val(x)
            if _ok_tensor(x, ac) and tuple(shape) == (xv.shape[-1],) \
                    and all(p is None or (_ok_tensor(p, ac, 1) and _val(p).dtype == xv.dtype) for p in (w, b)):
                self._replace(node, _layer_norm, (x, w, b, float(eps)), "layer_norm")
            return
        if _in(node, _RMSNORM):
            x, shape = node.args[:2]
            w = _arg(node, 2, "weight")
            eps = _arg(node, 3, "eps")
            xv = _val(x)
            if eps is not None and _ok_tensor(x, ac) and tuple(shape) == (xv.shape[-1],) \
                    and (w is None or (_ok_tensor(w, ac, 1) and _val(w).dtype == xv.dtype)):
                self._replace(node, _rms_norm, (x, w, float(eps)), "rms_norm")
            return
        if _in(node, _ROWRED):
            kind = _ROWRED[t]
            x = node.args[0]
            dim = _arg(node, 1, "dim")
            keep = _arg(node, 2, "keepdim", False)
            xv = _val(x)
            if _ok_tensor(x, ac) and _is_last_dim(dim, xv) and not keep and node.kwargs.get("dtype") is None \
                    and xv.dim() >= 1 and xv.shape[-1] > 0:
                self._replace(node, _rowred, (x, kind), f"row_{kind}")
            elif _ok_tensor(x, ac) and not keep and node.kwargs.get("dtype") is None and xv.dim() >= 2:
                # one other axis: the middle-axis reduction
                d = dim[0] if isinstance(dim, (list, tuple)) and len(dim) == 1 else dim
                if isinstance(d, int) and -xv.dim() <= d < xv.dim() and xv.shape[d] > 0:
                    self._replace(node, _axisred, (x, kind, int(d)), f"reduce_{kind}(dim)")
            return

    def _attn_weights_ok(self, E, H, *ps) -> bool:
        ac = self.allow_cpu
        if not isinstance(E, int) or not isinstance(H, int) or H <= 0 or E % H or E // H > 128:
            return False
        return all(p is None or _ok_tensor(p, ac) for p in ps)

    def _visit_mha_functional(self, node: fx.Node):
        a = node.args
        if len(a) < 13:
            return
        q, k, v, E, H, w_in, b_in, bias_k, bias_v, add_zero, drop, w_out, b_out = a[:13]
        kw = node.kwargs
        if bias_k is not None or bias_v is not None or add_zero or kw.get("need_weights", True):
            return
        if kw.get("training", True) and drop not in (0, 0.0):
            return
        if kw.get("key_padding_mask") is not None or kw.get("attn_mask") is not None:
            return
        if kw.get("use_separate_proj_weight", False) or kw.get("static_k") is not None \
                or kw.get("static_v") is not None:
            return
        causal = bool(kw.get("is_causal", False))
        if causal:
            return  # is_causal without a mask is a hint only in this function
        ac = self.allow_cpu
        if not all(_ok_tensor(x, ac, 3) for x in (q, k, v)):
            return
        qv, kv, vv = _val(q), _val(k), _val(v)
        if not (qv.shape == kv.shape == vv.shape and qv.dtype == kv.dtype == vv.dtype):
            return
        if not self._attn_weights_ok(E, H, w_in, b_in, w_out, b_out) or w_in is None or w_out is None:
            return
        self._replace(node, _mha_functional, (q, k, v, H, w_in, b_in, w_out, b_out, False), "attention(mha)")

    def _visit_mha_native(self, node: fx.Node):
        a = node.args
        if len(a) < 9:
            return
        q, k, v, E, H, w_in, b_in, w_out, b_out = a[:9]
        mask = a[9] if len(a) > 9 else node.kwargs.get("mask")
        need_w = a[10] if len(a) > 10 else node.kwargs.get("need_weights", True)
        if mask is not None or need_w:
            return
        ac = self.allow_cpu
        if not all(_ok_tensor(x, ac, 3) for x in (q, k, v)):
            return
        qv, kv, vv = _val(q), _val(k), _val(v)
        if not (qv.shape == kv.shape == vv.shape and qv.dtype == kv.dtype == vv.dtype):
            return
        if not self._attn_weights_ok(E, H, w_in, b_in, w_out, b_out):
            return
        self._replace(node, _mha_native, (q, k, v, H, w_in, b_in, w_out, b_out), "attention(mha)")

    def _visit_encoder_layer(self, node: fx.Node):
        a = node.args
        if len(a) < 18:
            return
        x, E, H, w_in, b_in, w_out, b_out, use_gelu, norm_first, eps = a[:10]
        n1w, n1b, n2w, n2b, l1w, l1b, l2w, l2b = a[10:18]
        mask = a[18] if len(a) > 18 else node.kwargs.get("mask")
        if mask is not None or not _ok_tensor(x, self.allow_cpu, 3):
            return
        if not self._attn_weights_ok(E, H, w_in, b_in, w_out, b_out, n1w, n1b, n2w, n2b,
                                     l1w, l1b, l2w, l2b):
            return
        self._replace(node, _encoder_layer, (x, H, w_in, b_in, w_out, b_out, bool(use_gelu),
                                             bool(norm_first), float(eps), n1w, n1b, n2w, n2b,
                                             l1w, l1b, l2w, l2b), "encoder_layer")

    def _explicit_attention(self, out_mm: fx.Node, sm: fx.Node, v) -> bool:
        if not _is_last_dim(_arg(sm, 1, "dim"), _val(sm)):
            return False
        s = sm.args[0]
        scale = 1.0
        if isinstance(s, fx.Node) and _target_key(s) in (operator.mul, torch.mul, "mul", operator.truediv, torch.div, "div") \
                and len(s.users) == 1:
            x, c = s.args
            if isinstance(c, fx.Node) or not isinstance(c, (int, float)):
                return False
            scale = float(c) if _target_key(s) in (operator.mul, torch.mul, "mul") else 1.0 / float(c)
            s = x
        if not (isinstance(s, fx.Node) and _in(s, _MATMUL) and len(s.users) == 1):
            return False
        q, kt = s.args
        if not (isinstance(kt, fx.Node) and _target_key(kt) in (torch.transpose, "transpose")):
            return False
        k = kt.args[0]
        dims = tuple(d % 4 for d in kt.args[1:3]) if len(kt.args) >= 3 else ()
        if sorted(dims) != [2, 3]:
            return False
        if not all(_ok_tensor(x, self.allow_cpu, 4) for x in (q, k, v)):
            return False
        qv, kv, vv = _val(q), _val(k), _val(v)
        if not (qv.shape == kv.shape == vv.shape and qv.dtype == kv.dtype == vv.dtype and qv.shape[-1] <= 128):
            return False
        self._replace(out_mm, _sdpa, (q, k, v, False, scale), "attention(explicit)")
        return True


def rewrite(gm: fx.GraphModule, allow_cpu: bool = False) -> List[str]:
    """Rewrite ``gm`` in place; returns the tags of the replaced patterns."""
    return Rewriter(gm, allow_cpu).run()


# Tags of the patterns replaced in the most recent graph (last_rewrites) and in
# every graph compiled since the caller last cleared it (rewrite_log; one
# torch.compile call can produce several graphs when Dynamo breaks the graph).
last_rewrites: List[str] = []
rewrite_log: List[str] = []


def b2msl_backend(gm: fx.GraphModule, example_inputs, inner: str = "eager"):
    """Dynamo backend: rewrite the hot-path patterns, then run eagerly or via Inductor."""
    global last_rewrites
    last_rewrites = rewrite(gm)
    rewrite_log.extend(last_rewrites)
    if inner == "inductor":
        from torch._inductor.compile_fx import compile_fx
        return compile_fx(gm, example_inputs)
    return gm.forward


def register() -> None:
    """Register ``backend="b2msl"`` (and ``"b2msl_inductor"``) with torch.compile."""
    from torch._dynamo import register_backend
    from torch._dynamo.backends.registry import _BACKENDS
    if "b2msl" not in _BACKENDS:
        register_backend(name="b2msl")(b2msl_backend)
    if "b2msl_inductor" not in _BACKENDS:
        register_backend(name="b2msl_inductor")(
            lambda gm, ex: b2msl_backend(gm, ex, inner="inductor"))
