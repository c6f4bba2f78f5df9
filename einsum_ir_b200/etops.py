"""Tensor operations from explicit descriptors, on the B200 backend.

The public surface of the reference's ``etops`` package
(python/src/etops/__init__.py:1-567 over the pybind11 module
python/src/bindings.cpp:14-334): ``TensorOperationConfig`` (dimension types,
execution types, sizes and a [LEVEL][TENSOR][DIMENSION] stride tensor, with
the same validation and JSON form), ``TensorOperation`` (set-up + execute),
``optimize`` and the enum namespaces ``prim``, ``exec`` / ``etype``, ``dim``,
``float32`` / ``float64``. A configuration written for the reference runs
unchanged: ``backend="tpp"`` (or None) selects this backend.

The operation is set up through the C-ABI (include/eir_tensor_operation.h)
and runs on the GPU: a binary contraction (prim_main gemm / brgemm) on the
tcgen05, DMMA or CUDA-core kernels the planner picks, a unary copy or zero on
the permute kernels. Execution types and level-1 packing strides are
accepted with the reference's shape rules; they describe CPU scheduling and
do not change the result. ``execute`` takes CUDA tensors (run in place on
the current stream) or host arrays / CPU tensors (staged through device
memory, the output written back in place). Unlike the reference, every
operand is checked against the extent its strides address.
"""
from __future__ import annotations

import ctypes
import enum
import json
from ctypes import byref, c_int32, c_int64, c_void_p
from dataclasses import dataclass
from typing import Dict, Optional, Sequence, Union

from . import cabi


class DataType(enum.IntEnum):
    float32 = 0
    float64 = 1


class PrimType(enum.IntEnum):
    none = 0
    zero = 1
    copy = 2
    relu = 3
    gemm = 4
    brgemm = 5


class ExecType(enum.IntEnum):
    seq = 0
    prim = 1
    shared = 2
    sfc = 3


class DimType(enum.IntEnum):
    c = 0
    m = 1
    n = 2
    k = 3


class ErrorType(enum.IntEnum):
    success = 0
    compilation_failed = 1
    invalid_stride_shape = 2
    invalid_optimization_config = 3


dtype = DataType
float32 = DataType.float32
float64 = DataType.float64

_BACKENDS = (None, "tpp", "b200")
_OPT_KEYS = ("target_m", "target_n", "target_k", "num_threads", "br_gemm_support",
             "packed_gemm_support", "packing_support", "sfc_support", "l2_cache_size")
_BOOL_KEYS = ("br_gemm_support", "packed_gemm_support", "packing_support", "sfc_support")


class prim:
    """primitive types"""
    none = PrimType.none
    zero = PrimType.zero
    relu = PrimType.relu
    copy = PrimType.copy
    gemm = PrimType.gemm
    brgemm = PrimType.brgemm


class etype:
    """execution types"""
    prim = ExecType.prim
    seq = ExecType.seq
    shared = ExecType.shared
    sfc = ExecType.sfc


exec = etype  # noqa: A001  (the reference's name)


class dim:
    """dimension types"""
    c = DimType.c
    m = DimType.m
    n = DimType.n
    k = DimType.k


def _is_binary(p) -> bool:
    return p in (PrimType.gemm, PrimType.brgemm)


def _is_unary(p) -> bool:
    return p in (PrimType.copy, PrimType.zero)


def _err_name(e: int) -> str:
    try:
        return f"ErrorType.{ErrorType(e).name}"
    except ValueError:
        return f"ErrorType({e})"


@dataclass(frozen=True)
class TensorOperationConfig:
    """Configuration of one binary contraction or unary operation.

    strides: [LEVEL][TENSOR][DIMENSION]; level 0 = memory layout (binary:
    in0, in1, out; unary: in, out), level 1 = packing (accepted, not needed
    on the GPU). Validation as the reference's __post_init__
    (python/src/etops/__init__.py:150-246).
    """
    data_type: DataType
    prim_first: PrimType
    prim_main: PrimType
    prim_last: PrimType
    dim_types: Sequence[DimType]
    exec_types: Sequence[ExecType]
    dim_sizes: Sequence[int]
    strides: Sequence[Sequence[Sequence[int]]]
    backend: Optional[str] = None

    def __post_init__(self):
        if self.backend not in _BACKENDS:
            raise ValueError(f"Unsupported backend: '{self.backend}'. Supported: 'tpp' (this backend), 'b200'.")
        binary, unary = _is_binary(self.prim_main), _is_unary(self.prim_main)
        if not binary and not unary:
            raise ValueError(f"Invalid prim_main: {self.prim_main}. Must be gemm/brgemm (binary) or copy/zero (unary).")
        nd = len(self.dim_types)
        if len(self.exec_types) != nd:
            raise ValueError(f"exec_types length ({len(self.exec_types)}) must match dim_types length ({nd}).")
        if len(self.dim_sizes) != nd:
            raise ValueError(f"dim_sizes length ({len(self.dim_sizes)}) must match dim_types length ({nd}).")
        for i, s in enumerate(self.dim_sizes):
            if s <= 0:
                raise ValueError(f"dim_sizes[{i}] must be positive, got {s}.")
        if len(self.strides) == 0:
            raise ValueError("strides must have at least one level (level 0).")
        want = 3 if binary else 2
        names = ["in0", "in1", "out"] if binary else ["in", "out"]
        if len(self.strides[0]) != want:
            raise ValueError(f"strides[0] must have {want} tensors ({', '.join(names)}), got {len(self.strides[0])}.")
        for t, v in enumerate(self.strides[0]):
            if len(v) != nd:
                raise ValueError(f"strides[0][{t}] ({names[t]}) length ({len(v)}) must match number of dimensions ({nd}).")
        if unary:
            for i, d in enumerate(self.dim_types):
                if d != DimType.c:
                    raise ValueError(f"For unary operations, all dim_types must be etops.dim.c. dim_types[{i}] is {d!r}.")
            if self.prim_first != PrimType.none:
                raise ValueError(f"For unary operations, prim_first must be etops.prim.none, got {self.prim_first!r}.")
            if self.prim_last != PrimType.none:
                raise ValueError(f"For unary operations, prim_last must be etops.prim.none, got {self.prim_last!r}.")
        else:
            if self.prim_first not in (PrimType.none, PrimType.zero):
                raise ValueError("For binary contractions, prim_first must be etops.prim.none or "
                                 f"etops.prim.zero, got {self.prim_first!r}.")
            if self.prim_last not in (PrimType.none, PrimType.relu):
                raise ValueError("For binary contractions, prim_last must be etops.prim.none or "
                                 f"etops.prim.relu, got {self.prim_last!r}.")

    def apply(self, op: "TensorOperation") -> None:
        """set up `op` with this configuration (RuntimeError on failure)"""
        err = op.setup(self.backend or "tpp", self.data_type, self.prim_first, self.prim_main,
                       self.prim_last, tuple(self.dim_types), tuple(self.exec_types),
                       tuple(self.dim_sizes),
                       tuple(tuple(tuple(t) for t in level) for level in self.strides))
        if err != ErrorType.success:
            raise RuntimeError(f"einsum_ir TensorOperation setup failed: {_err_name(err)}")

    def to_json(self, indent: Optional[int] = None) -> str:
        data = {
            "data_type": DataType(self.data_type).name,
            "prim_first": PrimType(self.prim_first).name,
            "prim_main": PrimType(self.prim_main).name,
            "prim_last": PrimType(self.prim_last).name,
            "dim_types": [DimType(d).name for d in self.dim_types],
            "exec_types": [ExecType(e).name for e in self.exec_types],
            "dim_sizes": list(self.dim_sizes),
            "strides": [[list(t) for t in level] for level in self.strides],
        }
        if self.backend is not None:
            data["backend"] = self.backend
        return json.dumps(data, indent=indent)

    @classmethod
    def from_json(cls, json_str: str) -> "TensorOperationConfig":
        data = json.loads(json_str)
        required = ["data_type", "prim_first", "prim_main", "prim_last", "dim_types", "exec_types",
                    "dim_sizes", "strides"]
        missing = [f for f in required if f not in data]
        if missing:
            raise ValueError(f"Missing required fields: {missing}")

        def get(enum_type, name):
            try:
                return enum_type[name]
            except KeyError:
                raise ValueError(f"Invalid {enum_type.__name__} value: '{name}'") from None

        return cls(data_type=get(DataType, data["data_type"]),
                   prim_first=get(PrimType, data["prim_first"]),
                   prim_main=get(PrimType, data["prim_main"]),
                   prim_last=get(PrimType, data["prim_last"]),
                   dim_types=tuple(get(DimType, d) for d in data["dim_types"]),
                   exec_types=tuple(get(ExecType, e) for e in data["exec_types"]),
                   dim_sizes=tuple(data["dim_sizes"]),
                   strides=tuple(tuple(tuple(t) for t in level) for level in data["strides"]),
                   backend=data.get("backend"))

    def save(self, path: str, indent: Optional[int] = 2) -> None:
        with open(path, "w") as f:
            f.write(self.to_json(indent=indent))

    @classmethod
    def load(cls, path: str) -> "TensorOperationConfig":
        with open(path) as f:
            return cls.from_json(f.read())


def _flat_strides(strides):
    """[LEVEL][TENSOR][DIMENSION] -> (levels, tensors per level, dims per vector, flat) ctypes arrays"""
    tpl, dpv, flat = [], [], []
    for level in strides:
        tpl.append(len(level))
        for v in level:
            dpv.append(len(v))
            flat.extend(int(x) for x in v)
    mk = lambda t, xs: (t * max(1, len(xs)))(*xs)
    return len(tpl), mk(c_int32, tpl), mk(c_int32, dpv), mk(c_int64, flat)


def _descriptor(dim_types, exec_types, dim_sizes):
    n = len(dim_sizes)
    return (n, (c_int32 * max(1, n))(*[int(d) for d in dim_types]),
            (c_int32 * max(1, n))(*[int(e) for e in exec_types]),
            (c_int64 * max(1, n))(*[int(s) for s in dim_sizes]))


class _OptConfig(ctypes.Structure):
    _fields_ = [("target_m", c_int64), ("target_n", c_int64), ("target_k", c_int64),
                ("num_threads", c_int64), ("br_gemm_support", c_int32),
                ("packed_gemm_support", c_int32), ("packing_support", c_int32),
                ("sfc_support", c_int32), ("l2_cache_size", c_int64)]


class TensorOperation:
    """One set-up tensor operation (the reference's _etops_core.TensorOperation
    wrapped by etops.TensorOperation)."""

    def __init__(self, config: Optional[TensorOperationConfig] = None):
        L = cabi.lib()
        self._h = c_void_p()
        cabi.check(L.eir_top_create(byref(self._h)))
        self._cfg = None
        if config is not None:
            config.apply(self)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            cabi.lib().eir_top_destroy(h)
            self._h = c_void_p()

    def setup(self, backend, dtype, prim_first, prim_main, prim_last, dim_types, exec_types, dim_sizes,
              strides) -> ErrorType:
        """set-up (bindings.cpp:54-105); returns an ErrorType"""
        if backend not in ("tpp", "b200"):
            return ErrorType.compilation_failed
        n, dt, et, ds = _descriptor(dim_types, exec_types, dim_sizes)
        nl, tpl, dpv, flat = _flat_strides(strides)
        err = ErrorType(cabi.lib().eir_top_setup(self._h, int(dtype), int(prim_first), int(prim_main),
                                                  int(prim_last), n, dt, et, ds, nl, tpl, dpv, flat))
        self._cfg = (DataType(dtype), PrimType(prim_main), tuple(int(s) for s in dim_sizes),
                     [tuple(int(x) for x in v) for v in strides[0]]) if err == ErrorType.success else None
        return err

    # ---- execution
    def execute(self, in0, in1, out) -> None:
        """out <- op(in0, in1); in1 is None for unary operations (bindings.cpp:107-131)"""
        if self._cfg is None:
            raise RuntimeError("einsum_ir TensorOperation: execute before a successful setup")
        import numpy as np
        import torch
        dt, pm, sizes, strides0 = self._cfg
        binary = _is_binary(pm)
        tdt = torch.float64 if dt == DataType.float64 else torch.float32
        if binary and in1 is None:
            raise ValueError("binary contraction: in1 is required")
        operands = [in0, in1] if binary else [in0]
        out_strides = strides0[2] if binary else strides0[1]
        np_dt = np.float64 if tdt == torch.float64 else np.float32

        def fits(x, st, name):
            numel = x.numel() if isinstance(x, torch.Tensor) else np.asarray(x).size
            lo = sum((s - 1) * min(v, 0) for s, v in zip(sizes, st))
            hi = sum((s - 1) * max(v, 0) for s, v in zip(sizes, st))
            if lo < 0 or hi >= numel:
                raise ValueError(f"{name}: strides address elements {lo}..{hi} but the operand holds {numel}")

        # every check before any device work
        for i, x in enumerate(operands):
            fits(x, strides0[i], f"in{i}" if binary else "in")
        fits(out, out_strides, "out")
        if isinstance(out, torch.Tensor):
            if out.dtype != tdt or not out.is_contiguous():
                raise ValueError(f"out must be a contiguous {tdt} tensor")
        elif not isinstance(out, np.ndarray) or out.dtype != np_dt or not out.flags.c_contiguous \
                or not out.flags.writeable:
            raise ValueError("out must be a writable C-contiguous array of the configured data type")
        on_device = isinstance(out, torch.Tensor) and out.is_cuda
        dev = out.device if on_device else torch.device("cuda", torch.cuda.current_device())
        dev_in = []
        for x in operands:
            if isinstance(x, torch.Tensor):
                dev_in.append(x.to(device=dev, dtype=tdt).contiguous())
            else:
                dev_in.append(torch.from_numpy(np.ascontiguousarray(x, dtype=np_dt)).to(dev))
        if on_device:
            dout = out
        elif isinstance(out, torch.Tensor):
            dout = out.to(dev)
        else:
            dout = torch.from_numpy(out).to(dev)
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev)
            cabi.check(cabi.lib().eir_top_execute(self._h, c_void_p(dev_in[0].data_ptr()),
                                                   c_void_p(dev_in[1].data_ptr() if binary else None),
                                                   c_void_p(dout.data_ptr()), c_void_p(stream.cuda_stream)))
            if not on_device:
                host = dout.cpu()
                if isinstance(out, torch.Tensor):
                    out.copy_(host)
                else:
                    np.copyto(out, host.numpy())

    # ---- extensions of this backend
    @property
    def plan(self) -> cabi.Plan:
        """a view of the operation's plan (valid while the operation lives)"""
        h = cabi.lib().eir_top_plan(self._h)
        if not h:
            raise RuntimeError("einsum_ir TensorOperation: not set up")
        return cabi.Plan(c_void_p(h), owned=False)

    def describe(self) -> str:
        h = cabi.lib().eir_top_plan(self._h)
        return cabi.lib().eir_plan_describe(c_void_p(h)).decode() if h else "not set up"

    @staticmethod
    def get_default_optimization_config(backend: str = "tpp") -> Dict[str, Union[int, bool]]:
        c = _OptConfig()
        cabi.check(cabi.lib().eir_top_default_optimization_config(byref(c)))
        return {k: (bool(getattr(c, k)) if k in _BOOL_KEYS else int(getattr(c, k))) for k in _OPT_KEYS}

    @staticmethod
    def optimize(backend, dtype, prim_first, prim_main, prim_last, dim_types, exec_types, dim_sizes,
                 strides, optimization_config: Dict) -> tuple:
        """(error, dtype, prim_first, prim_main, prim_last, dim_types, exec_types, dim_sizes,
        strides) as the reference's static optimize (bindings.cpp:133-250)"""
        fail = lambda e: (e, dtype, prim_first, prim_main, prim_last, dim_types, exec_types,
                          dim_sizes, [])
        if backend not in ("tpp", "b200"):
            return fail(ErrorType.compilation_failed)
        cfg = _OptConfig(**{k: v for k, v in TensorOperation.get_default_optimization_config().items()})
        try:
            for key, val in optimization_config.items():
                if key not in _OPT_KEYS:
                    return fail(ErrorType.invalid_optimization_config)
                if key in _BOOL_KEYS:
                    if not isinstance(val, (bool, int)):
                        raise TypeError(key)
                    setattr(cfg, key, int(bool(val)))
                else:
                    if isinstance(val, bool) or not isinstance(val, int):
                        raise TypeError(key)
                    setattr(cfg, key, int(val))
        except (TypeError, AttributeError):
            return fail(ErrorType.invalid_optimization_config)
        n, dt, et, ds = _descriptor(dim_types, exec_types, dim_sizes)
        nl, tpl, dpv, flat = _flat_strides(strides)
        cap = max(1, n)
        o_n, o_t = c_int32(0), c_int32(0)
        o_dt, o_et = (c_int32 * cap)(), (c_int32 * cap)()
        o_ds, o_st = (c_int64 * cap)(), (c_int64 * (3 * cap))()
        err = ErrorType(cabi.lib().eir_top_optimize(int(dtype), int(prim_first), int(prim_main),
                                                     int(prim_last), n, dt, et, ds, nl, tpl, dpv, flat,
                                                     byref(cfg), byref(o_n), o_dt, o_et, o_ds, byref(o_t),
                                                     o_st))
        if err != ErrorType.success:
            return fail(err)
        m = o_n.value
        level = tuple(tuple(o_st[t * m + i] for i in range(m)) for t in range(o_t.value))
        return (err, DataType(dtype), PrimType(prim_first), PrimType(prim_main), PrimType(prim_last),
                tuple(DimType(o_dt[i]) for i in range(m)), tuple(ExecType(o_et[i]) for i in range(m)),
                tuple(o_ds[i] for i in range(m)), (level,))


class _B200Backend:
    """the tensor operation backend of this package (also selected by 'tpp')"""
    name: str = "tpp"

    @staticmethod
    def get_default_optimization_config() -> Dict[str, Union[int, bool]]:
        return TensorOperation.get_default_optimization_config("tpp")


class backend:
    """available backends"""
    tpp = _B200Backend()
    b200 = _B200Backend()


def optimize(config: TensorOperationConfig,
             optimization_config: Optional[Dict[str, Union[int, bool]]] = None) -> TensorOperationConfig:
    """optimised configuration (python/src/etops/__init__.py:467-547): for this
    backend, size-1 dims dropped, dims contiguous in every tensor fused, and
    execution types naming how the GPU kernels run the loops"""
    actual = config.backend if config.backend is not None else "tpp"
    if optimization_config is None:
        if actual in ("tpp", "b200"):
            optimization_config = backend.tpp.get_default_optimization_config()
        else:
            raise ValueError(f"Unknown backend: {actual}")
    r = TensorOperation.optimize(actual, config.data_type, config.prim_first, config.prim_main,
                                 config.prim_last, tuple(config.dim_types), tuple(config.exec_types),
                                 tuple(config.dim_sizes),
                                 tuple(tuple(tuple(t) for t in level) for level in config.strides),
                                 optimization_config)
    err = r[0]
    if err != ErrorType.success:
        raise RuntimeError(f"einsum_ir optimization failed: {_err_name(err)}")
    return TensorOperationConfig(backend=actual, data_type=r[1], prim_first=r[2], prim_main=r[3],
                                 prim_last=r[4], dim_types=r[5], exec_types=r[6], dim_sizes=r[7],
                                 strides=r[8])


__all__ = ["TensorOperation", "TensorOperationConfig", "DataType", "PrimType", "ExecType", "DimType",
           "dtype", "float32", "float64", "prim", "etype", "exec", "dim", "backend", "optimize",
           "ErrorType"]
