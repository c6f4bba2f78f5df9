"""GPU permute (Unary COPY) parity: bit-exact against the oracle.

Mirrors the reference's unary tests (UnaryTpp.test.torch.cpp:5-199): 2-D
transposes, higher-order permutations, identity copies, for every element
size the path moves (BF16 = 2 bytes, FP32 = 4, FP64 = 8).
"""
import itertools

import numpy as np
import pytest

from einsum_ir_b200 import cabi
from tests import _oracle

pytestmark = pytest.mark.gpu

ESIZE = {cabi.BF16: 2, cabi.FP32: 4, cabi.FP64: 8}
NPDT = {2: np.uint16, 4: np.uint32, 8: np.uint64}


def row_major(shape):
    s, out = 1, []
    for n in reversed(shape):
        out.append(s)
        s *= n
    return list(reversed(out))


def run_perm(cuda, shape, perm, dtype, seed=0):
    import torch
    es = ESIZE[dtype]
    rng = np.random.default_rng(seed)
    n = int(np.prod(shape)) if shape else 1
    src = rng.integers(0, 2 ** (8 * es) - 1, size=n, dtype=np.uint64).astype(NPDT[es])
    out_shape = [shape[p] for p in perm]
    sin = row_major(shape)
    sout_perm = row_major(out_shape)
    sout = [0] * len(shape)
    for j, p in enumerate(perm):
        sout[p] = sout_perm[j]
    plan = cabi.PermutePlan(shape, sin, sout, dtype)
    tdt = {2: torch.int16, 4: torch.int32, 8: torch.int64}[es]
    d_src = torch.from_numpy(src.view({2: np.int16, 4: np.int32, 8: np.int64}[es])).to(cuda)
    d_dst = torch.zeros(n, dtype=tdt, device=cuda)
    plan.permute(d_src, d_dst)
    torch.cuda.synchronize()
    got = d_dst.cpu().numpy().view(NPDT[es])
    ref = np.zeros(n, dtype=NPDT[es])
    _oracle.permute(shape, sin, sout, es, src, ref)
    assert np.array_equal(got, ref), f"{shape} {perm} {plan.describe()}"


SHAPES = [(64, 128), (33, 65), (3, 5, 7, 11), (2, 3, 4, 5, 6), (128, 4, 96), (1, 17, 1, 9)]


@pytest.mark.parametrize("dtype", [cabi.BF16, cabi.FP32, cabi.FP64])
@pytest.mark.parametrize("shape", SHAPES)
def test_permute_all_perms(cuda, shape, dtype):
    perms = list(itertools.permutations(range(len(shape))))
    if len(perms) > 24:
        rng = np.random.default_rng(1)
        perms = [perms[i] for i in rng.choice(len(perms), 24, replace=False)] + [tuple(range(len(shape)))]
    for p in perms:
        run_perm(cuda, list(shape), list(p), dtype)


def test_permute_large_transpose(cuda):
    run_perm(cuda, [1024, 2048], [1, 0], cabi.FP32)
    run_perm(cuda, [512, 64, 32], [0, 2, 1], cabi.BF16)


def test_permute_empty(cuda):
    run_perm(cuda, [0, 5], [1, 0], cabi.FP32)
