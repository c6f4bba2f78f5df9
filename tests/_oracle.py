"""Test-side binding of the CPU oracle (oracle/eir_oracle.c).

The oracle is test infrastructure: this helper is imported only by tests,
__graft_entry__.smoke() and bench.py's CPU-baseline leg.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_int32, c_int64, c_void_p
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "_build" / "libeir_oracle.so"
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
        L = ctypes.CDLL(str(LIB))
        L.eir_oracle_contract.argtypes = [c_int32, POINTER(c_int32)] + [POINTER(c_int64)] * 5 + \
            [c_int32] * 6 + [c_void_p] * 4 + [c_int32]
        L.eir_oracle_permute.argtypes = [c_int32] + [POINTER(c_int64)] * 3 + [c_int32, c_void_p, c_void_p]
        L.eir_oracle_round_tf32.argtypes = [c_void_p, c_void_p, c_int64]
        _lib = L
    return _lib


def _arr(ctype, vals):
    return (ctype * max(1, len(vals)))(*vals)


def _p(a):
    return None if a is None else c_void_p(a.ctypes.data)


def contract(dims, left, right, out, aux=None, dt_l=0, dt_r=0, dt_o=0, comp=0,
             first=0, last=99, threads=0):
    """In-place oracle contraction. dims: (type, size, sl, sr, so, sa) tuples.
    Arrays are flat numpy buffers (BF16 data as uint16 bit patterns)."""
    n = len(dims)
    rc = lib().eir_oracle_contract(
        n, _arr(c_int32, [d[0] for d in dims]), _arr(c_int64, [d[1] for d in dims]),
        _arr(c_int64, [d[2] for d in dims]), _arr(c_int64, [d[3] for d in dims]),
        _arr(c_int64, [d[4] for d in dims]), _arr(c_int64, [d[5] for d in dims]),
        dt_l, dt_r, dt_o, comp, first, last, _p(left), _p(right), _p(aux), _p(out), threads)
    assert rc == 0


def permute(sizes, sin, sout, esize, src, dst):
    n = len(sizes)
    rc = lib().eir_oracle_permute(n, _arr(c_int64, sizes), _arr(c_int64, sin), _arr(c_int64, sout),
                                  esize, _p(src), _p(dst))
    assert rc == 0


def round_tf32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().eir_oracle_round_tf32(_p(x), _p(y), x.size)
    return y


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    den = np.linalg.norm(b)
    num = np.linalg.norm(a - b)
    return float(num / den) if den > 0 else float(num)
