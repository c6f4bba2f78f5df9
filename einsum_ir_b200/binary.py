"""Python front door for strided binary contractions over the C-ABI.

Mirrors the reference's ``backend::BinaryContraction`` interface
(src/backend/BinaryContraction.h:16-392): dimension types are derived from
the dimension ids of the left, right and output tensors
(BinaryContraction.cpp:7-111), strides are row-major from the outer sizes with
stride 0 for dims of size < 2 (BinaryContraction.cpp:223-249), and
``num_ops`` counts 2*|C||M||N||K| minus |C||M||N| for a ZERO first touch
(BinaryContraction.cpp:434-465). ``contract`` takes device pointers (or torch
CUDA tensors) and runs asynchronously on the given stream.
"""
from __future__ import annotations

from typing import Dict, List, Mapping, Optional, Sequence, Tuple

from . import cabi

C, M, N, K, I, J = 0, 1, 2, 3, 5, 6
UNDEFINED_DIM = 99


def _types_of(t0: Sequence[int], t1: Sequence[int], t2: Sequence[int],
              only2: int, with0: int, with1: int, with01: int) -> List[int]:
    """Type of every dim of t2 relative to t0 and t1 (BinaryContraction.cpp:7-61)."""
    s0, s1 = set(t0), set(t1)
    out = []
    for d in t2:
        a, b = d in s0, d in s1
        out.append(with01 if (a and b) else with0 if a else with1 if b else only2)
    return out


def dim_types(ids_left: Sequence[int], ids_right: Sequence[int], ids_out: Sequence[int]
              ) -> Tuple[List[int], List[int], List[int]]:
    """(left, right, out) dim types as in BinaryContraction::dim_types (:63-111)."""
    left = _types_of(ids_right, ids_out, ids_left, I, K, M, C)
    right = _types_of(ids_left, ids_out, ids_right, J, K, N, C)
    out = _types_of(ids_left, ids_right, ids_out, UNDEFINED_DIM, M, N, C)
    return left, right, out


def dim_types_ids(ids_left, ids_right, ids_out) -> Dict[str, List[int]]:
    """C/M/N from the output order, K/I from the left order, J from the right (:131-221)."""
    tl, tr, to = dim_types(ids_left, ids_right, ids_out)
    return {
        "c": [d for d, t in zip(ids_out, to) if t == C],
        "m": [d for d, t in zip(ids_out, to) if t == M],
        "n": [d for d, t in zip(ids_out, to) if t == N],
        "k": [d for d, t in zip(ids_left, tl) if t == K],
        "i": [d for d, t in zip(ids_left, tl) if t == I],
        "j": [d for d, t in zip(ids_right, tr) if t == J],
    }


def strides(ids: Sequence[int], sizes: Mapping[int, int]) -> Dict[int, int]:
    """Row-major strides from outer sizes; size < 2 gives stride 0 (:223-249)."""
    res: Dict[int, int] = {}
    s = 1
    for d in reversed(list(ids)):
        res[d] = 0 if sizes[d] < 2 else s
        s *= sizes[d]
    return res


def swap_inputs(ids_left, ids_right, ids_out) -> bool:
    """True if the output's fastest dim is N (or C with N before M), BinaryPrimitives.cpp:87-134."""
    _, _, to = dim_types(ids_left, ids_right, ids_out)
    if not to:
        return False
    if to[-1] == N:
        return True
    if to[-1] == C:
        for t in reversed(to):
            if t == M:
                return False
            if t == N:
                return True
    return False


def contraction_dims(ids_left, ids_right, ids_out, sizes_inner: Mapping[int, int],
                     sizes_outer_left=None, sizes_outer_right=None, sizes_outer_out=None,
                     sizes_outer_aux=None, cpx_id=None) -> List[tuple]:
    """eir_dim tuples (type, size, stride_left, stride_right, stride_out, stride_aux).
    cpx_id: id of the complex dim (size 2, in all three tensors) -> type DIM_CPX."""
    sl = strides(ids_left, sizes_outer_left or sizes_inner)
    sr = strides(ids_right, sizes_outer_right or sizes_inner)
    so = strides(ids_out, sizes_outer_out or sizes_inner)
    sa = strides(ids_out, sizes_outer_aux) if sizes_outer_aux is not None else so
    g = dim_types_ids(ids_left, ids_right, ids_out)
    if g["i"] or g["j"]:
        raise ValueError("I/J dims (summed over one operand only) are not supported")
    dims = []
    for t, key in ((C, "c"), (M, "m"), (N, "n"), (K, "k")):
        for d in g[key]:
            ty = cabi.DIM_CPX if d == cpx_id else t
            dims.append((ty, int(sizes_inner[d]), sl.get(d, 0), sr.get(d, 0),
                         so.get(d, 0) if t != K else 0, sa.get(d, 0) if t != K else 0))
    return dims


def parse_binary(expr: str) -> Tuple[List[int], List[int], List[int], List[str]]:
    """'akmj,njk->anm' -> dim ids (names sorted, EinsumExpressionAscii.cpp:267-303)."""
    lhs, out = expr.replace(" ", "").split("->")
    left, right = lhs.split(",")
    names = sorted(set(left + right + out))
    idx = {c: i for i, c in enumerate(names)}
    return [idx[c] for c in left], [idx[c] for c in right], [idx[c] for c in out], names


class BinaryContraction:
    """init/compile/contract/num_ops over eir_contract_plan_create / eir_contract."""

    def init(self, ids_left, ids_right, ids_out, sizes_inner, sizes_outer_left=None,
             sizes_outer_right=None, sizes_outer_aux=None, sizes_outer_out=None,
             dtype_left=cabi.FP32, dtype_right=cabi.FP32, dtype_comp=cabi.COMPUTE_DEFAULT,
             dtype_out=cabi.FP32, ktype_first_touch=cabi.KTYPE_ZERO,
             ktype_main=cabi.KTYPE_MADD, ktype_last_touch=cabi.KTYPE_UNDEFINED, flags=0):
        self.dims = contraction_dims(ids_left, ids_right, ids_out, sizes_inner,
                                     sizes_outer_left, sizes_outer_right, sizes_outer_out,
                                     sizes_outer_aux)
        g = dim_types_ids(ids_left, ids_right, ids_out)
        self.dim_ids = g
        self.sizes = {k: [int(sizes_inner[d]) for d in v] for k, v in g.items()}
        self._args = (dtype_left, dtype_right, dtype_out, dtype_comp, ktype_first_touch,
                      ktype_main, ktype_last_touch, flags)
        self.plan: Optional[cabi.ContractPlan] = None

    def compile(self) -> int:
        dl, dr, do, dc, f, m, l, fl = self._args
        self.plan = cabi.ContractPlan(self.dims, dl, dr, do, dc, f, m, l, fl)
        return cabi.SUCCESS

    def contract(self, left, right, out, aux=None, stream: int = 0) -> None:
        if self.plan is None:
            raise cabi.EirError(5, "called before compilation")
        self.plan.contract(left, right, out, aux, stream)

    def num_ops(self) -> int:
        return self.plan.num_ops if self.plan else 0
