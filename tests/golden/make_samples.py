"""Writes tests/golden/samples/: seeded synthetic setting files in the line
formats of the reference's sample suites (samples/**/*.cfg: an expression
line ``"expression" "sizes" "path"`` and a tree line ``"tree" "sizes"``), used
by tests/test_gpu_samples.py to run einsum_ir_b200.run_samples in every GPU
test run. The settings are random tensor networks of this generator, not the
suites' own items.

    python tests/golden/make_samples.py
"""
from __future__ import annotations

import random
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tests import _tree  # noqa: E402

OUT = Path(__file__).resolve().parent / "samples"
LETTERS = "abcdefghijklmnopqrstuvwxyz"


def network(rng: random.Random):
    """(input strings, output string, sizes by letter, path pairs)"""
    while True:
        n_t = rng.randint(3, 5)
        n_d = rng.randint(n_t + 2, 9)
        dims = list(LETTERS[:n_d])
        tensors = [[] for _ in range(n_t)]
        out = []
        for d in dims:
            kind = rng.random()
            if kind < 0.55:                       # contracted between two tensors
                a, b = rng.sample(range(n_t), 2)
                tensors[a].append(d)
                tensors[b].append(d)
            elif kind < 0.85:                     # free: one tensor and the output
                tensors[rng.randrange(n_t)].append(d)
                out.append(d)
            else:                                 # batch: two tensors and the output
                a, b = rng.sample(range(n_t), 2)
                tensors[a].append(d)
                tensors[b].append(d)
                out.append(d)
        if any(len(t) == 0 for t in tensors) or not out:
            continue
        for t in tensors:
            rng.shuffle(t)
        rng.shuffle(out)
        sizes = {d: rng.choice([2, 3, 4, 6, 8, 12, 16, 24, 32]) for d in dims}
        flops = 1
        for d in dims:
            flops *= sizes[d]
        if flops > 2 ** 28 or flops < 2 ** 12:
            continue
        pairs = [(0, 1)] * (n_t - 1)  # left to right
        return ["".join(t) for t in tensors], "".join(out), sizes, pairs


def tree_string(inputs, output, sizes, pairs):
    """the tree of the left-to-right path, intermediates by the reference's
    rules (tests/_tree.py), in the einsum-tree text format"""
    ids = {c: i for i, c in enumerate(sorted(sizes))}
    expr = ",".join(inputs) + "->" + output
    size_str = ",".join(str(sizes[c]) for c in sorted(sizes))
    path = ",".join(f"({a},{b})" for a, b in pairs)
    strings, _, pp = _tree.parse(expr, size_str, path)
    steps, tensors = _tree.tree_plan(strings, pp)
    text = {i: "[" + ",".join(str(d) for d in strings[i]) + "]" for i in range(len(inputs))}
    for c, (l, r, out) in enumerate(steps):
        node = f"{text[l]},{text[r]}->[{','.join(str(d) for d in out)}]"
        text[len(inputs) + c] = node if c == len(steps) - 1 else "[" + node + "]"
    return text[len(inputs) + len(steps) - 1], ",".join(str(sizes[c]) for c in sorted(sizes, key=ids.get))


def main():
    rng = random.Random(20261202)
    OUT.mkdir(exist_ok=True)
    expr_lines, tree_lines = [], []
    for _ in range(8):
        inputs, output, sizes, pairs = network(rng)
        expr = ",".join(inputs) + "->" + output
        size_str = ",".join(str(sizes[c]) for c in sorted(sizes))
        path = ",".join(f"({a},{b})" for a, b in pairs)
        expr_lines.append(f'"{expr}" "{size_str}" "{path}"')
        tree, tsizes = tree_string(inputs, output, sizes, pairs)
        tree_lines.append(f'"{tree}" "{tsizes}"')
    (OUT / "synthetic.cfg").write_text("\n".join(expr_lines) + "\n")
    (OUT / "synthetic_et.cfg").write_text("\n".join(tree_lines) + "\n")
    print(f"wrote {len(expr_lines)} expression and {len(tree_lines)} tree settings to {OUT}")


if __name__ == "__main__":
    main()
