"""The CPU oracle reproduces the reference's own oracle outputs (golden fixtures
made by tests/golden/make_golden.py from the reference's test modules)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLD = np.load(Path(__file__).parent / "golden" / "golden.npz")
META = json.loads(bytes(GOLD["__meta__"]).decode())


def _t(name, key):
    return torch.from_numpy(GOLD[f"{name}/{key}"].copy())


@pytest.mark.parametrize("case", [m["name"] for m in META if m["name"].startswith("fa_")])
def test_attention_oracle_matches_reference(case):
    q, k, v, o = (_t(case, n) for n in "qkvo")
    causal = bool(_t(case, "causal").item())
    got = O.ref_attention(q, k, v, causal=causal)
    assert torch.equal(got, o.float()) or O.max_abs_err(got, o) < 1e-6


@pytest.mark.parametrize("form,fn", [("2d_sum_ax1", O.ref_sum), ("2d_max_ax1", O.ref_max),
                                     ("2d_argmax_ax1", O.ref_argmax)])
def test_reduce_oracle_matches_reference(form, fn):
    x, out = _t(f"reduce_{form}", "x"), _t(f"reduce_{form}", "out")
    got = fn(x)
    if form.endswith("argmax_ax1"):
        assert torch.equal(got, out.long())
    else:
        assert torch.allclose(got, out, equal_nan=True, atol=0, rtol=0)


def test_row_family_oracle_matches_reference():
    x = _t("softmax", "x")
    assert torch.allclose(O.ref_softmax(x), _t("softmax", "out"), atol=1e-7)
    w, b = _t("layernorm", "w"), _t("layernorm", "b")
    assert torch.allclose(O.ref_layernorm(x, w, b, 1e-5), _t("layernorm", "out"), atol=1e-6)
    assert torch.allclose(O.ref_rmsnorm(x, _t("rmsnorm", "w"), 1e-6), _t("rmsnorm", "out"), atol=1e-6)


def test_gemm_oracle_matches_reference():
    a, b, bias, out = (_t("gemm_bias_relu", k) for k in ("a", "b", "bias", "out"))
    got = O.ref_gemm(a, b, bias, "relu", torch.float32)
    assert O.max_abs_err(got, out) < 1e-5


def test_argmax_tie_and_nan_semantics():
    x = torch.tensor([[1.0, 3.0, 3.0], [float("nan"), 5.0, float("nan")], [2.0, 2.0, 2.0]])
    assert O.ref_argmax(x).tolist() == [1, 0, 0]
    assert O.ref_argmin(x).tolist() == [0, 0, 0]
