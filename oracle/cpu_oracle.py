"""ctypes binding of the C restatement (oracle/cpu_moe.c) -- test
infrastructure and CPU baseline only."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import build as _build
from .nvfp4_oracle import BankHost


class _Bank(C.Structure):
    _fields_ = [
        ("experts", C.c_int),
        ("hidden", C.c_int),
        ("intermediate", C.c_int),
        ("packed", C.c_void_p * 3),
        ("scales", C.c_void_p * 3),
        ("inv_scales", C.c_void_p),
        ("router", C.c_void_p),
        ("router_bias", C.c_void_p),
    ]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = C.CDLL(str(path))
        _lib.nvfp4_oracle_cpu_gemv.argtypes = [
            C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_int,
        ]
        _lib.nvfp4_oracle_cpu_gemv.restype = C.c_int
        _lib.nvfp4_oracle_moe_forward.argtypes = [
            C.POINTER(_Bank), C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
        ]
        _lib.nvfp4_oracle_moe_forward.restype = C.c_int
    return _lib


def cpu_gemv(packed: np.ndarray, scales: np.ndarray, x: np.ndarray, weight_global_scale: float,
             threads: int = 0) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    rows = packed.shape[0]
    out = np.empty(rows, dtype=np.float32)
    st = lib().nvfp4_oracle_cpu_gemv(packed.ctypes.data, scales.ctypes.data, rows, packed.shape[1] * 2,
                                     weight_global_scale, x.ctypes.data, out.ctypes.data, threads)
    if st:
        raise ValueError("invalid CPU GEMV arguments")
    return out


@dataclass
class DenseBank:
    """Contiguous host arrays of a full bank in the device layout."""

    experts: int
    hidden: int
    intermediate: int
    packed: list           # 3 x uint8 [(E+1)*rows*cols/2]
    scales: list           # 3 x uint8 [(E+1)*rows*cols/16]
    inv_scales: np.ndarray  # float32 [3, E+1]
    router: np.ndarray      # uint16 [(E+1), H]
    router_bias: np.ndarray | None = None

    @classmethod
    def from_host(cls, bank: BankHost) -> "DenseBank":
        E, H, I = bank.experts, bank.hidden, bank.intermediate
        packed, scales = [], []
        inv = np.zeros((3, E + 1), dtype=np.float32)
        for p in range(3):
            packed.append(np.concatenate([bank.projections[p][e].packed.reshape(-1) for e in range(E + 1)]))
            scales.append(np.concatenate([bank.projections[p][e].scales.reshape(-1) for e in range(E + 1)]))
            for e in range(E + 1):
                inv[p, e] = np.float32(1.0) / np.float32(bank.projections[p][e].global_scale)
        bias = None if bank.router_bias is None else np.ascontiguousarray(bank.router_bias, dtype=np.float32)
        return cls(E, H, I, packed, scales, inv, np.ascontiguousarray(bank.router_all()), bias)

    def _struct(self) -> _Bank:
        b = _Bank()
        b.experts, b.hidden, b.intermediate = self.experts, self.hidden, self.intermediate
        for p in range(3):
            b.packed[p] = self.packed[p].ctypes.data
            b.scales[p] = self.scales[p].ctypes.data
        b.inv_scales = self.inv_scales.ctypes.data
        b.router = self.router.ctypes.data
        b.router_bias = self.router_bias.ctypes.data if self.router_bias is not None else None
        return b

    def forward(self, x: np.ndarray, residual: np.ndarray | None = None, threads: int = 0):
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.empty((T, self.hidden), dtype=np.float32)
        ids = np.empty((T, 9), dtype=np.int32)
        weights = np.empty((T, 9), dtype=np.float32)
        logits = np.empty((T, self.experts + 1), dtype=np.float32)
        res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        st = lib().nvfp4_oracle_moe_forward(
            C.byref(self._struct()), x.ctypes.data, T, None if res is None else res.ctypes.data,
            out.ctypes.data, ids.ctypes.data, weights.ctypes.data, logits.ctypes.data, threads)
        if st:
            raise RuntimeError(f"CPU oracle forward failed ({st})")
        return out, ids, weights, logits


def route(router_all_bf16: np.ndarray, x: np.ndarray, router_bias: np.ndarray | None = None,
          threads: int | None = None):
    """Routing of T tokens by the C restatement (nvfp4_oracle_route): the
    same FP32 fixed-order logits and lowest-id top-8 as ``moe_layer``, fast
    enough for the 8192-token BASELINE calls. router_all_bf16 is [(E+1), H]
    BF16 bits with row E the shared gate; x is [T, H] float32. Returns (ids
    [T, 9] int32, weights [T, 9] float32, logits [T, E+1] float32)."""
    import os

    router = np.ascontiguousarray(router_all_bf16, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, H = router.shape
    E = R - 1
    T = x.shape[0]
    b = _Bank()
    b.experts, b.hidden, b.intermediate = E, H, 0
    b.router = router.ctypes.data
    bias = None if router_bias is None else np.ascontiguousarray(router_bias, dtype=np.float32)
    b.router_bias = None if bias is None else bias.ctypes.data
    ids = np.empty((T, 9), dtype=np.int32)
    weights = np.empty((T, 9), dtype=np.float32)
    logits = np.empty((T, R), dtype=np.float32)
    f = lib().nvfp4_oracle_route
    f.argtypes = [C.POINTER(_Bank), C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
    f.restype = C.c_int
    st = f(C.byref(b), x.ctypes.data, T, ids.ctypes.data, weights.ctypes.data, logits.ctypes.data,
           threads if threads is not None else (os.cpu_count() or 1))
    if st:
        raise ValueError("invalid routing arguments")
    return ids, weights, logits
