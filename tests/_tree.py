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


def contract_step(dims, a, b, n_out, model="fp64"):
    """one binary contraction of the oracle. model: "fp64" (FP64 values and
    intermediates), "fp32" (operands and result stored as FP32, as this
    backend's FP32 / BF16 trees store intermediates) or "tf32" (as fp32, with
    the operands rounded to TF32 first)"""
    if model == "fp64":
        res = np.zeros(n_out, dtype=np.float64)
        _oracle.contract(dims, np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel(), res, None,
                         cabi.FP64, cabi.FP64, cabi.FP64)
        return res
    res = np.zeros(n_out, dtype=np.float32)
    _oracle.contract(dims, np.asarray(a, np.float32).ravel(), np.asarray(b, np.float32).ravel(), res, None,
                     cabi.FP32, cabi.FP32, cabi.FP32, cabi.COMPUTE_TF32 if model == "tf32" else 0)
    return res


def eval_tree(expr, sizes, path, inputs, dtype=cabi.FP32, model="fp64"):
    strings, size_list, pairs = parse(expr, sizes, path)
    steps, tensors = tree_plan(strings, pairs)
    szmap = {i: s for i, s in enumerate(size_list)}
    vals = {i: np.asarray(inputs[i], dtype=np.float64).ravel() for i in range(len(strings) - 1)}
    n_in = len(strings) - 1
    for c, (l, r, out) in enumerate(steps):
        dims = binary.contraction_dims(tensors[l], tensors[r], out, szmap)
        n_out = int(np.prod([szmap[d] for d in out])) if out else 1
        vals[n_in + c] = contract_step(dims, vals[l], vals[r], n_out, model)
    return vals[n_in + len(steps) - 1]


def eval_nodes(nodes, sizes, leaves, model="fp64"):
    """A parsed einsum tree with the oracle: nodes[i] = (dim ids, children) in
    post order (children before their parent, the root last); a node with two
    children contracts them into its dims, one child is permuted into its
    dims; leaves maps a leaf's node index to its values."""
    vals = {}
    for i, (ids, ch) in enumerate(nodes):
        if not ch:
            vals[i] = np.asarray(leaves[i], dtype=np.float64).ravel()
        elif len(ch) == 1:
            src = nodes[ch[0]][0]
            sin = binary.strides(src, sizes)
            sout = binary.strides(ids, sizes)
            out = np.zeros(int(np.prod([sizes[d] for d in ids])) if ids else 1)
            _oracle.permute([sizes[d] for d in src], [sin[d] for d in src], [sout[d] for d in src], 8,
                            np.ascontiguousarray(vals[ch[0]], np.float64), out)
            vals[i] = out
        else:
            l, r = ch
            dims = binary.contraction_dims(nodes[l][0], nodes[r][0], ids, sizes)
            n_out = int(np.prod([sizes[d] for d in ids])) if ids else 1
            vals[i] = contract_step(dims, vals[l], vals[r], n_out, model)
    return vals[len(nodes) - 1]


def load_dump(d):
    """(manifest {key: value}, tensor(name) -> (ids, sizes, values)) of a
    driver's EIR_DRIVER_DUMP directory"""
    from pathlib import Path
    d = Path(d)
    man = {}
    for line in (d / "manifest.txt").read_text().splitlines():
        k, _, v = line.partition(" ")
        man[k] = v

    def tensor(name):
        f = man[name].split()
        ids = [] if f[1] == "-" else [int(x) for x in f[1].split(",")]
        sz = [] if f[3] == "-" else [int(x) for x in f[3].split(",")]
        return ids, sz, np.fromfile(d / f"{name}.f64", dtype=np.float64)
    return man, tensor
