"""Test-side tree evaluation with the CPU oracle (test infrastructure).

Restates the reference's tree construction (EinsumExpression.cpp:72-99 for
the unique path ids, :25-70 for the intermediate dims in ascending id order,
EinsumExpressionAscii.cpp:267-303 for the numeric-aware name order) and
evaluates each binary contraction with the C oracle in float64.
"""
from __future__ import annotations

import numpy as np

from einsum_ir_b200 import binary, cabi
from tests import _oracle


def parse(expr: str, sizes: str, path: str):
    lhs, out = expr.replace(" ", "").split("->")
    ins = lhs.split(",")
    names = sorted(set(lhs.replace(",", "") + out))
    ids = {c: i for i, c in enumerate(names)}
    strings = [[ids[c] for c in t] for t in ins] + [[ids[c] for c in out]]
    size_list = [int(s) for s in sizes.split(",")]
    pairs = [int(x) for x in path.replace("(", "").replace(")", "").replace(" ", "").split(",") if x]
    return strings, size_list, [(pairs[2 * i], pairs[2 * i + 1]) for i in range(len(pairs) // 2)]


def unique_ids(n_conts, path):
    live = list(range(n_conts + 1))
    nxt = n_conts + 1
    out = []
    for a, b in path:
        out.append((live[a], live[b]))
        for p in sorted((a, b), reverse=True):
            live.pop(p)
        live.append(nxt)
        nxt += 1
    return out


def tree_plan(strings, path):
    """[(left tensor id, right tensor id, out dims)] in evaluation order."""
    n_in = len(strings) - 1
    hist = {}
    for s in strings:
        for d in s:
            hist[d] = hist.get(d, 0) + 1
    tensors = {i: list(strings[i]) for i in range(n_in)}
    steps = []
    for c, (l, r) in enumerate(unique_ids(n_in - 1, path)):
        for d in tensors[l] + tensors[r]:
            hist[d] -= 1
        if c == len(path) - 1:
            out = list(strings[-1])
        else:
            out = sorted({d for d in tensors[l] + tensors[r] if hist[d] > 0})
            for d in out:
                hist[d] += 1
        tensors[n_in + c] = out
        steps.append((l, r, out))
    return steps, tensors


def eval_tree(expr, sizes, path, inputs, dtype=cabi.FP32):
    strings, size_list, pairs = parse(expr, sizes, path)
    steps, tensors = tree_plan(strings, pairs)
    szmap = {i: s for i, s in enumerate(size_list)}
    vals = {i: np.asarray(inputs[i], dtype=np.float64).ravel() for i in range(len(strings) - 1)}
    n_in = len(strings) - 1
    for c, (l, r, out) in enumerate(steps):
        dims = binary.contraction_dims(tensors[l], tensors[r], out, szmap)
        res = np.zeros(int(np.prod([szmap[d] for d in out])) if out else 1, dtype=np.float64)
        _oracle.contract(dims, vals[l], vals[r], res, None, cabi.FP64, cabi.FP64, cabi.FP64)
        vals[n_in + c] = res
    return vals[n_in + len(steps) - 1]
