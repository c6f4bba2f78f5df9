"""Generates the golden fixtures of tests/golden/ (run once; outputs committed).

The reference's numeric tests compare against at::einsum on random inputs
(e.g. EinsumExpression.test.torch.cpp:695-787, BinaryContractionTpp.test.torch.cpp);
there are no stored reference outputs. These fixtures freeze that check:
seeded inputs and the torch.einsum result in float64 (the same einsum
semantics as at::einsum), so later runs compare the oracle and the CUDA path
against fixed numbers. Cases: the README expression at the reference test's
sizes and path, reduced BASELINE configs 2-5, and a bias+ReLU MLP layer.

    python tests/golden/make_golden.py
"""
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = [
    # name, expression, sizes by sorted dim name, path (opt_einsum pairs) or None, dtype
    ("readme_tree", "iae,bf,dcba,cg,dh->hgfei", dict(a=4, b=3, c=5, d=8, e=7, f=2, g=3, h=6, i=9),
     [(1, 2), (2, 3), (0, 1), (0, 1)], "fp32"),
    ("readme_tree_fp64", "iae,bf,dcba,cg,dh->hgfei", dict(a=4, b=3, c=5, d=8, e=7, f=2, g=3, h=6, i=9),
     [(1, 2), (2, 3), (0, 1), (0, 1)], "fp64"),
    ("cfg2_binary_bf16", "akmj,njk->anm", dict(a=2, k=4, m=128, j=64, n=128), None, "bf16"),
    ("cfg4_tucker", "abc,ia,jb,kc->ijk", dict(a=8, b=8, c=8, i=16, j=16, k=16),
     [(0, 1), (0, 2), (0, 1)], "fp32"),
    ("cfg5_batch_fp64", "zabcd,zcdef->zabef", dict(z=2, a=4, b=4, c=4, d=4, e=4, f=4), None, "fp64"),
]


def make_case(name, expr, sizes, path, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    lhs, out = expr.split("->")
    ins = lhs.split(",")
    tdt = {"fp64": torch.float64, "bf16": torch.bfloat16}.get(dtype, torch.float32)
    tens = [(torch.rand([sizes[c] for c in t], generator=g, dtype=torch.float64) * 2 - 1).to(tdt)
            for t in ins]
    ref = torch.einsum(expr, *[t.double() for t in tens])
    arrs = {}
    for i, t in enumerate(tens):
        arrs[f"in{i}"] = t.view(torch.int16).numpy().view(np.uint16) if tdt == torch.bfloat16 else t.numpy()
    arrs["out"] = ref.numpy()
    meta = dict(expr=expr, sizes=",".join(str(sizes[c]) for c in sorted(sizes)),
                path="" if path is None else ",".join(f"({a},{b})" for a, b in path), dtype=dtype)
    np.savez_compressed(HERE / f"{name}.npz", **arrs, **{k: np.array(v) for k, v in meta.items()})


def make_mlp(seed=5):
    # one hidden layer of bench_mlp (bench_mlp.cpp:207-290): out[b,o] = relu(sum_i x[b,i] w[i,o] + bias[o])
    g = torch.Generator().manual_seed(seed)
    b, i, o = 64, 96, 80
    x = torch.rand(b, i, generator=g, dtype=torch.float64) * 2 - 1
    w = torch.randn(i, o, generator=g, dtype=torch.float64) / i ** 0.5
    bias = torch.rand(o, generator=g, dtype=torch.float64) * 2 - 1
    x, w, bias = x.float(), w.float(), bias.float()
    ref = torch.relu(x.double() @ w.double() + bias.double())
    np.savez_compressed(HERE / "cfg3_mlp_layer.npz", x=x.numpy(), w=w.numpy(), bias=bias.numpy(),
                        out=ref.numpy())


if __name__ == "__main__":
    for k, case in enumerate(CASES):
        make_case(*case, seed=100 + k)
    make_mlp()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
