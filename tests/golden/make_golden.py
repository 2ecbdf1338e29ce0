"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/triton-msl

It imports the reference's OWN oracle functions from its test modules
(`_ref_attention` in tests/test_flash_attention.py:124-135, `_ref` in
tests/test_fa_simdgroup_diff.py:18-24, `_ref` in tests/test_fuzz_reduce.py:100-139)
and records their outputs on seeded inputs. Where the reference writes the
oracle inline in a test body (softmax tests/test_integration.py:552, RMS
:1081-1082, LayerNorm :1124, matmul tests/test_fast_matmul_parity.py:53 and
tests/test_matmul_epilogue.py:80), the expression is evaluated here verbatim
and the fixture records which line it came from. The output is
tests/golden/golden.npz (small; committed). Nothing at test time reads the
reference checkout.
"""
from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden.npz"


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(Path(ref_root) / "tests"))
    tfa = importlib.import_module("test_flash_attention")
    tdiff = importlib.import_module("test_fa_simdgroup_diff")
    tred = importlib.import_module("test_fuzz_reduce")

    arrays: dict[str, np.ndarray] = {}
    meta: list[dict] = []

    def put(name, source, **tensors):
        for k, v in tensors.items():
            arrays[f"{name}/{k}"] = v.detach().cpu().numpy()
        meta.append({"name": name, "source": source, "keys": sorted(tensors)})

    # FlashAttention, fp32, through _ref_attention (its scale is 1/sqrt(D)).
    for (n, d, causal) in [(50, 32, False), (100, 64, True), (128, 64, False), (192, 128, True),
                           (64, 128, False)]:
        g = torch.Generator().manual_seed(1000 + n + d)
        q = torch.randn(1, 1, n, d, generator=g)
        k = torch.randn(1, 1, n, d, generator=g)
        v = torch.randn(1, 1, n, d, generator=g)
        o = tfa._ref_attention(q, k, v, causal=causal)
        put(f"fa_f32_n{n}_d{d}_c{int(causal)}", "tests/test_flash_attention.py:124-135",
            q=q, k=k, v=v, o=o, causal=torch.tensor(int(causal)))

    # FlashAttention, fp16 inputs upcast, through test_fa_simdgroup_diff._ref.
    for (n, d, causal) in [(128, 128, True), (100, 128, False), (50, 64, True)]:
        g = torch.Generator().manual_seed(2000 + n + d)
        q = torch.randn(1, 1, n, d, generator=g).half()
        k = torch.randn(1, 1, n, d, generator=g).half()
        v = torch.randn(1, 1, n, d, generator=g).half()
        o = tdiff._ref(q, k, v, causal)
        put(f"fa_f16_n{n}_d{d}_c{int(causal)}", "tests/test_fa_simdgroup_diff.py:18-24",
            q=q, k=k, v=v, o=o, causal=torch.tensor(int(causal)))

    # Row reductions through test_fuzz_reduce._ref, including ties and NaN rows.
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 300, generator=g)
    x[3, :] = 1.0                     # all-tie row -> argmax 0
    x[5, 17] = x[5, 200] = 50.0       # two-way tie -> lower index
    x[7, 123] = float("nan")          # NaN row
    x[9, 10] = x[9, 250] = float("nan")
    for form in ("2d_sum_ax1", "2d_max_ax1", "2d_argmax_ax1"):
        r = tred._ref(form, x)
        put(f"reduce_{form}", "tests/test_fuzz_reduce.py:100-139", x=x, out=r)

    # Inline oracle expressions of the reference tests, evaluated verbatim.
    xs = torch.randn(16, 1000, generator=g)
    put("softmax", "tests/test_integration.py:552 torch.softmax(x, dim=1)",
        x=xs, out=torch.softmax(xs, dim=1))
    w = torch.randn(1000, generator=g) * 0.1 + 1.0
    b = torch.randn(1000, generator=g) * 0.1
    put("layernorm", "tests/test_integration.py:1124 torch.layer_norm",
        x=xs, w=w, b=b, out=torch.layer_norm(xs, [1000], w, b, 1e-5))
    rms = xs / torch.sqrt(torch.mean(xs * xs, dim=-1, keepdim=True) + 1e-6) * w
    put("rmsnorm", "tests/test_integration.py:1081-1082", x=xs, w=w, out=rms)
    a = torch.randn(64, 48, generator=g)
    bm = torch.randn(48, 80, generator=g)
    bias = torch.randn(80, generator=g) * 0.3
    put("gemm_bias_relu", "tests/test_fast_matmul_parity.py:53 + tests/test_matmul_epilogue.py:80",
        a=a, b=bm, bias=bias,
        out=torch.from_numpy(np.maximum((a.float() @ bm.float()).numpy() + bias.numpy()[None, :], 0.0)))

    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(meta)} cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to a triton-msl checkout>")
    main(sys.argv[1])
