"""ctypes binding of the C-ABI declared in include/eir_cuda.h.

The library is loaded from this package directory (built in-tree by
``einsum_ir_b200.build``). There is no fallback: if the shared library is
missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int32, c_int64, c_void_p
from pathlib import Path
from typing import Iterable, Sequence

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libeinsum_ir_b200.so"

# ---- enums (values of include/eir_cuda.h)
SUCCESS = 0
DIM_C, DIM_M, DIM_N, DIM_K, DIM_CPX = 0, 1, 2, 3, 4
FP32, FP64, BF16 = 0, 1, 2
COMPUTE_DEFAULT, COMPUTE_FP32, COMPUTE_TF32, COMPUTE_FP64, COMPUTE_BF16 = 0, 1, 2, 3, 4
KTYPE_ZERO, KTYPE_RELU, KTYPE_ADD, KTYPE_COPY, KTYPE_MADD, KTYPE_UNDEFINED = 0, 1, 2, 3, 4, 99
KTYPE_CPX_ZERO, KTYPE_CPX_MADD = 6, 8
FAMILY_NONE, FAMILY_SIMT, FAMILY_TC, FAMILY_PERMUTE, FAMILY_DMMA = 0, 1, 2, 3, 4
FLAG_FORCE_SIMT, FLAG_NO_PREPACK = 1, 2

# every symbol include/eir_cuda.h declares (checked by the CPU test suite)
EXPORTS = [
    "eir_contract_plan_create", "eir_contract", "eir_contract_num_ops",
    "eir_permute_plan_create", "eir_permute", "eir_plan_destroy", "eir_plan_kernel_family",
    "eir_plan_workspace_bytes", "eir_plan_describe", "eir_expression_create",
    "eir_expression_eval", "eir_expression_num_ops", "eir_expression_num_tensors",
    "eir_expression_tensor_dims", "eir_expression_destroy", "eir_expression_describe",
    "eir_last_error_string", "eir_check_device_errors", "eir_launch_count", "eir_version",
    "eir_plan_profile", "eir_plan_profile_read", "eir_contract_no_alloc", "eir_unary_plan_create",
    "eir_contract_peers", "eir_ipc_get_handle", "eir_ipc_open_handle", "eir_ipc_close_handle",
    "eir_copy_to_peers", "eir_contract_gather", "eir_output_group_create", "eir_output_group_peers",
    "eir_output_group_destroy",
    # include/eir_tensor_operation.h
    "eir_top_create", "eir_top_destroy", "eir_top_setup", "eir_top_execute", "eir_top_plan",
    "eir_top_default_optimization_config", "eir_top_optimize",
]


class EirDim(ctypes.Structure):
    _fields_ = [("type", c_int32), ("pad_", c_int32), ("size", c_int64),
                ("stride_left", c_int64), ("stride_right", c_int64),
                ("stride_out", c_int64), ("stride_out_aux", c_int64)]


class EirContractDesc(ctypes.Structure):
    _fields_ = [("num_dims", c_int32), ("dtype_left", c_int32), ("dtype_right", c_int32),
                ("dtype_out", c_int32), ("dtype_comp", c_int32),
                ("ktype_first_touch", c_int32), ("ktype_main", c_int32),
                ("ktype_last_touch", c_int32), ("flags", c_int32), ("pad_", c_int32),
                ("dims", POINTER(EirDim))]


class EirError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"einsum_ir_b200 error {code}: {msg}")
        self.code = code


_lib = None

# int (*)(void const *send, void *recv, int64_t bytes, void *user)
ALLGATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int, c_void_p, c_void_p, c_int64, c_void_p)


def lib() -> ctypes.CDLL:
    """Load the shared library once (raises if it is missing)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise EirError(-1, f"{LIB_PATH} missing: run einsum_ir_b200.build.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        L.eir_contract_plan_create.argtypes = [POINTER(EirContractDesc), POINTER(c_void_p)]
        L.eir_contract.argtypes = [c_void_p] * 6
        L.eir_contract_no_alloc.argtypes = [c_void_p] * 6
        L.eir_contract_peers.argtypes = [c_void_p] * 5 + [c_int32, POINTER(c_void_p), c_void_p]
        L.eir_contract_gather.argtypes = [c_void_p] * 5 + [c_int32, POINTER(c_void_p), c_void_p]
        L.eir_output_group_create.argtypes = [c_int32, c_int32, c_void_p, ALLGATHER_FN, c_void_p,
                                              POINTER(c_void_p)]
        L.eir_output_group_peers.argtypes = [c_void_p, c_int64, POINTER(c_void_p)]
        L.eir_output_group_destroy.argtypes = [c_void_p]
        L.eir_ipc_get_handle.argtypes = [c_void_p, c_void_p, POINTER(c_int64)]
        L.eir_ipc_open_handle.argtypes = [c_void_p, c_int64, POINTER(c_void_p), POINTER(c_void_p)]
        L.eir_ipc_close_handle.argtypes = [c_void_p]
        L.eir_copy_to_peers.argtypes = [c_void_p, c_int32, POINTER(c_void_p), c_int64, c_void_p]
        L.eir_contract_num_ops.argtypes = [c_void_p]
        L.eir_contract_num_ops.restype = c_int64
        L.eir_permute_plan_create.argtypes = [c_int32, POINTER(c_int64), POINTER(c_int64),
                                              POINTER(c_int64), c_int32, POINTER(c_void_p)]
        L.eir_permute.argtypes = [c_void_p] * 4
        L.eir_unary_plan_create.argtypes = [c_int32, POINTER(c_int64), POINTER(c_int64),
                                            POINTER(c_int64), c_int32, c_int32, POINTER(c_void_p)]
        L.eir_top_create.argtypes = [POINTER(c_void_p)]
        L.eir_top_destroy.argtypes = [c_void_p]
        L.eir_top_setup.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32,
                                    POINTER(c_int32), POINTER(c_int32), POINTER(c_int64), c_int32,
                                    POINTER(c_int32), POINTER(c_int32), POINTER(c_int64)]
        L.eir_top_execute.argtypes = [c_void_p] * 5
        L.eir_top_plan.argtypes = [c_void_p]
        L.eir_top_plan.restype = c_void_p
        L.eir_top_default_optimization_config.argtypes = [c_void_p]
        L.eir_top_optimize.argtypes = [c_int32, c_int32, c_int32, c_int32, c_int32,
                                       POINTER(c_int32), POINTER(c_int32), POINTER(c_int64), c_int32,
                                       POINTER(c_int32), POINTER(c_int32), POINTER(c_int64), c_void_p,
                                       POINTER(c_int32), POINTER(c_int32), POINTER(c_int32),
                                       POINTER(c_int64), POINTER(c_int32), POINTER(c_int64)]
        L.eir_plan_destroy.argtypes = [c_void_p]
        L.eir_plan_kernel_family.argtypes = [c_void_p]
        L.eir_plan_workspace_bytes.argtypes = [c_void_p]
        L.eir_plan_workspace_bytes.restype = c_int64
        L.eir_plan_describe.argtypes = [c_void_p]
        L.eir_plan_describe.restype = c_char_p
        L.eir_last_error_string.restype = c_char_p
        L.eir_check_device_errors.argtypes = [c_void_p]
        L.eir_launch_count.restype = c_int64
        L.eir_plan_profile.argtypes = [c_void_p, c_int32]
        L.eir_plan_profile_read.argtypes = [c_void_p, POINTER(ctypes.c_double), POINTER(c_int64)]
        if hasattr(L, "eir_expression_create"):
            L.eir_expression_create.argtypes = [c_char_p, c_char_p, c_char_p, c_int32, c_int32,
                                                 POINTER(c_void_p)]
            L.eir_expression_eval.argtypes = [c_void_p, POINTER(c_void_p), c_void_p]
            L.eir_expression_num_ops.argtypes = [c_void_p]
            L.eir_expression_num_ops.restype = c_int64
            L.eir_expression_num_tensors.argtypes = [c_void_p]
            L.eir_expression_tensor_dims.argtypes = [c_void_p, c_int32, POINTER(c_int64), c_int32]
            L.eir_expression_destroy.argtypes = [c_void_p]
            L.eir_expression_describe.argtypes = [c_void_p]
            L.eir_expression_describe.restype = c_char_p
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != SUCCESS:
        raise EirError(rc, lib().eir_last_error_string().decode())


def launch_count() -> int:
    return int(lib().eir_launch_count())


def check_device_errors(stream: int = 0) -> None:
    check(lib().eir_check_device_errors(c_void_p(stream)))


def _ptr(x) -> c_void_p:
    if x is None:
        return c_void_p(None)
    if isinstance(x, int):
        return c_void_p(x)
    if hasattr(x, "data_ptr"):
        return c_void_p(x.data_ptr())
    raise TypeError(f"cannot take a device pointer of {type(x)}")


class Plan:
    """A plan handle. owned=False: a view of a plan that another object owns
    (closing the view does not destroy the plan)."""

    def __init__(self, handle: c_void_p, owned: bool = True):
        self._h = handle
        self._owned = owned

    @property
    def handle(self) -> c_void_p:
        return self._h

    @property
    def family(self) -> int:
        return int(lib().eir_plan_kernel_family(self._h))

    @property
    def workspace_bytes(self) -> int:
        return int(lib().eir_plan_workspace_bytes(self._h))

    def describe(self) -> str:
        return lib().eir_plan_describe(self._h).decode()

    def profile(self, enable: bool = True) -> None:
        check(lib().eir_plan_profile(self._h, 1 if enable else 0))

    def profile_read(self) -> tuple:
        """(summed main-kernel milliseconds, timed launches) since the last read."""
        ms = ctypes.c_double()
        n = c_int64()
        check(lib().eir_plan_profile_read(self._h, ctypes.byref(ms), ctypes.byref(n)))
        return float(ms.value), int(n.value)

    def close(self) -> None:
        if self._h and self._owned:
            lib().eir_plan_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ContractPlan(Plan):
    """A compiled strided binary contraction (eir_contract_plan_create)."""

    def __init__(self, dims: Sequence[tuple], dtype_left: int, dtype_right: int, dtype_out: int,
                 dtype_comp: int = COMPUTE_DEFAULT, first: int = KTYPE_ZERO,
                 main: int = KTYPE_MADD, last: int = KTYPE_UNDEFINED, flags: int = 0):
        arr = (EirDim * max(1, len(dims)))()
        for i, d in enumerate(dims):
            t, size, sl, sr, so, sa = d
            arr[i] = EirDim(t, 0, size, sl, sr, so, sa)
        desc = EirContractDesc(len(dims), dtype_left, dtype_right, dtype_out, dtype_comp,
                               first, main, last, flags, 0, arr)
        h = c_void_p()
        check(lib().eir_contract_plan_create(ctypes.byref(desc), ctypes.byref(h)))
        super().__init__(h)
        self.dims = list(dims)

    @property
    def num_ops(self) -> int:
        return int(lib().eir_contract_num_ops(self._h))

    def contract(self, left, right, out, aux=None, stream: int = 0) -> None:
        check(lib().eir_contract(self._h, _ptr(left), _ptr(right), _ptr(aux), _ptr(out),
                                 c_void_p(stream)))

    def contract_no_alloc(self, left, right, out, aux=None, stream: int = 0) -> None:
        """eir_contract_no_alloc: same result, scratch from the library's static array."""
        check(lib().eir_contract_no_alloc(self._h, _ptr(left), _ptr(right), _ptr(aux), _ptr(out),
                                          c_void_p(stream)))

    def contract_peers(self, left, right, out, peer_outs: Sequence, aux=None, stream: int = 0) -> None:
        """eir_contract_peers: out and every peer output (device pointers or
        tensors with out's layout) receive the result."""
        ptrs = [_ptr(p) for p in peer_outs]
        arr = (c_void_p * max(1, len(ptrs)))(*ptrs)
        check(lib().eir_contract_peers(self._h, _ptr(left), _ptr(right), _ptr(aux), _ptr(out),
                                       len(ptrs), arr, c_void_p(stream)))

    def contract_gather(self, left, right, out, peer_outs: Sequence, aux=None, stream: int = 0) -> None:
        """eir_contract_gather: the contraction, then copy-engine copies of
        the output into every peer buffer (device pointers with out's extent),
        slab by slab as the kernel finishes them where the plan allows."""
        ptrs = [_ptr(p) for p in peer_outs]
        arr = (c_void_p * max(1, len(ptrs)))(*ptrs)
        check(lib().eir_contract_gather(self._h, _ptr(left), _ptr(right), _ptr(aux), _ptr(out),
                                        len(ptrs), arr, c_void_p(stream)))


IPC_HANDLE_BYTES = 64


class OutputGroup:
    """eir_output_group: every rank's full output buffer mapped into this
    process. `allgather(data: bytes) -> list[bytes]` (one entry per rank, in
    rank order) is the caller's exchange between the ranks; creation is
    collective."""

    def __init__(self, rank: int, world: int, out, allgather):
        def cb(send, recv, nbytes, user):
            try:
                parts = allgather(ctypes.string_at(send, nbytes))
                ctypes.memmove(recv, b"".join(parts), nbytes * world)
                return 0
            except Exception:
                return 1
        self._cb = ALLGATHER_FN(cb)  # kept alive while the library may call it
        self.world, self.rank = world, rank
        h = c_void_p()
        check(lib().eir_output_group_create(rank, world, _ptr(out), self._cb, None, ctypes.byref(h)))
        self._h = h

    def peers(self, offset: int) -> list:
        """addresses in the other ranks' buffers of byte `offset` of this rank's buffer"""
        arr = (c_void_p * max(1, self.world - 1))()
        check(lib().eir_output_group_peers(self._h, int(offset), arr))
        return [int(arr[i] or 0) for i in range(self.world - 1)]

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().eir_output_group_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ipc_get_handle(dev_ptr) -> tuple:
    """(handle bytes, offset) of a device pointer for another process of the node"""
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = c_int64()
    check(lib().eir_ipc_get_handle(_ptr(dev_ptr), h, ctypes.byref(off)))
    return bytes(h.raw), int(off.value)


def ipc_open_handle(handle: bytes, offset: int) -> tuple:
    """(device pointer, mapping base) of another process's buffer"""
    ptr, base = c_void_p(), c_void_p()
    check(lib().eir_ipc_open_handle(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), offset,
                                    ctypes.byref(ptr), ctypes.byref(base)))
    return int(ptr.value), int(base.value)


def ipc_close_handle(base: int) -> None:
    check(lib().eir_ipc_close_handle(c_void_p(base)))


def copy_to_peers(src, dsts: Sequence, nbytes: int, stream: int = 0) -> None:
    """copy-engine copies of nbytes from src to every destination pointer"""
    arr = (c_void_p * max(1, len(dsts)))(*[_ptr(d) for d in dsts])
    check(lib().eir_copy_to_peers(_ptr(src), len(dsts), arr, int(nbytes), c_void_p(stream)))


class PermutePlan(Plan):
    """A compiled permute (eir_permute_plan_create)."""

    def __init__(self, sizes: Sequence[int], strides_in: Sequence[int],
                 strides_out: Sequence[int], dtype: int):
        n = len(sizes)
        a = (c_int64 * max(1, n))(*sizes)
        b = (c_int64 * max(1, n))(*strides_in)
        c = (c_int64 * max(1, n))(*strides_out)
        h = c_void_p()
        check(lib().eir_permute_plan_create(n, a, b, c, dtype, ctypes.byref(h)))
        super().__init__(h)

    def permute(self, src, dst, stream: int = 0) -> None:
        check(lib().eir_permute(self._h, _ptr(src), _ptr(dst), c_void_p(stream)))


class Expression:
    """An einsum expression compiled into a tree of contractions (eir_expression_*)."""

    def __init__(self, expr: str, sizes: str, path: str, dtype: int = FP32,
                 dtype_comp: int = COMPUTE_DEFAULT):
        h = c_void_p()
        check(lib().eir_expression_create(expr.encode(), sizes.encode(), path.encode(), dtype,
                                          dtype_comp, ctypes.byref(h)))
        self._h = h

    @property
    def num_ops(self) -> int:
        return int(lib().eir_expression_num_ops(self._h))

    @property
    def num_tensors(self) -> int:
        return int(lib().eir_expression_num_tensors(self._h))

    def tensor_shape(self, i: int) -> list[int]:
        buf = (c_int64 * 64)()
        n = lib().eir_expression_tensor_dims(self._h, i, buf, 64)
        if n < 0:
            check(-n)
        return [int(buf[j]) for j in range(n)]

    def describe(self) -> str:
        return lib().eir_expression_describe(self._h).decode()

    def eval(self, tensors: Iterable, stream: int = 0) -> None:
        ptrs = [(_ptr(t).value or 0) for t in tensors]
        arr = (c_void_p * len(ptrs))(*ptrs)
        check(lib().eir_expression_eval(self._h, arr, c_void_p(stream)))

    def close(self) -> None:
        if self._h:
            lib().eir_expression_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
