"""Test-side binding of the reference's own scalar backends
(oracle/_ref/libref_scalar.so, built by oracle/ref.mk from the reference
sources). Test infrastructure: imported only by tests/ and bench.py's
CPU-baseline leg. available() is False when the library was not built (the
reference checkout was absent at build time)."""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_int32, c_int64, c_void_p
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "_ref" / "libref_scalar.so"
_lib = None


def available() -> bool:
    return LIB.exists()


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(LIB))
        L.ref_scalar_create.argtypes = [c_int64] * 3 + [POINTER(c_int64)] * 3 + [c_int64] + \
            [POINTER(c_int64)] * 3 + [c_int32] * 4 + [c_int64, POINTER(c_int32)]
        L.ref_scalar_create.restype = c_void_p
        L.ref_scalar_contract.argtypes = [c_void_p] * 5
        L.ref_scalar_num_ops.argtypes = [c_void_p]
        L.ref_scalar_num_ops.restype = c_int64
        L.ref_scalar_destroy.argtypes = [c_void_p]
        L.ref_scalar_permute.argtypes = [c_int64] + [POINTER(c_int64)] * 4 + [c_int32, c_void_p, c_void_p]
        L.ref_scalar_permute.restype = c_int32
        _lib = L
    return _lib


def _a(vals):
    return (c_int64 * max(1, len(vals)))(*vals)


def _p(a):
    return None if a is None else c_void_p(a.ctypes.data)


class Contraction:
    """backend::BinaryContractionScalar of the reference, compiled once.
    Tensors are row-major in the order of their dim ids; `sizes` maps every
    dim id to its size; `aux_outer` (None: no aux) maps dim ids to the aux
    tensor's outer sizes (1 = broadcast)."""

    def __init__(self, ids_l, ids_r, ids_o, sizes: dict, dtype=0, first=99, main=4, last=99,
                 aux_outer: dict | None = None, threads: int = 0):
        ids = sorted(sizes)
        err = c_int32(0)
        threads = threads if threads > 0 else (os.cpu_count() or 1)
        self._h = lib().ref_scalar_create(
            len(ids_l), len(ids_r), len(ids_o), _a(ids_l), _a(ids_r), _a(ids_o), len(ids), _a(ids),
            _a([sizes[i] for i in ids]), None if aux_outer is None else _a([aux_outer[i] for i in ids]),
            dtype, first, main, last, threads, ctypes.byref(err))
        if not self._h:
            raise RuntimeError(f"reference compile failed: err_t {err.value}")

    @property
    def num_ops(self) -> int:
        return int(lib().ref_scalar_num_ops(self._h))

    def contract(self, left: np.ndarray, right: np.ndarray, out: np.ndarray, aux: np.ndarray | None = None):
        for a in (left, right, out) + ((aux,) if aux is not None else ()):
            assert a.flags.c_contiguous
        lib().ref_scalar_contract(self._h, _p(left), _p(right), _p(aux), _p(out))

    def close(self):
        if self._h:
            lib().ref_scalar_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def permute(ids_in, ids_out, sizes: dict, src: np.ndarray, dst: np.ndarray, dtype=0) -> None:
    """backend::UnaryScalar (COPY) of the reference."""
    ids = sorted(sizes)
    rc = lib().ref_scalar_permute(len(ids_in), _a(ids_in), _a(ids_out), _a(ids),
                                  _a([sizes[i] for i in ids]), dtype, _p(src), _p(dst))
    assert rc == 0, rc
