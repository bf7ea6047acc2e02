"""Thin ctypes ownership layer over libnvfp4_moe_cuda.so (sm_100a).

Mirrors the lab's ``vllm_nvfp4_opencl/runtime.py``: the same classes
(``Profile``, ``TraceEvent``, ``DeviceBuffer``, ``MoeBank``, ``Runtime``), the
same method names, argument meaning and error behaviour
(``RuntimeError(f"{op} failed ({status}): {message}")``, runtime.py:820-823),
and the same process-wide ``get_runtime()`` singleton behind a lock
(runtime.py:1964-1976). There is no CPU execution path: when the CUDA
library or an sm_100a device is missing, construction raises.

Additions over the lab surface are marked "additive" and cover BF16 batched
forwards on torch tensors, routing introspection and device-side uploads.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np

LIB_NAME = "libnvfp4_moe_cuda.so"
NVFP4_MOE_ADD_RESIDUAL = 1
NVFP4_MOE_PARTIAL_F32 = 2
NVFP4_MOE_PRE_NORM = 4
NVFP4_DECODE_KERNELS_TENSOR_CORE = 0
NVFP4_DECODE_KERNELS_IN_REGISTER = 1
NVFP4_DECODE_KERNELS_FUSED_TOKEN = 2


class Profile(C.Structure):
    _fields_ = [
        ("upload_ns", C.c_uint64),
        ("kernel_ns", C.c_uint64),
        ("download_ns", C.c_uint64),
    ]


class _NativeTraceEvent(C.Structure):
    _fields_ = [
        ("scope", C.c_char * 96),
        ("operation", C.c_char * 64),
        ("queued_ns", C.c_uint64),
        ("submit_ns", C.c_uint64),
        ("start_ns", C.c_uint64),
        ("end_ns", C.c_uint64),
    ]


class _DeviceInfo(C.Structure):
    _fields_ = [
        ("platform_name", C.c_char * 256),
        ("device_name", C.c_char * 256),
        ("device_version", C.c_char * 256),
        ("driver_version", C.c_char * 256),
        ("global_memory_bytes", C.c_uint64),
        ("max_allocation_bytes", C.c_uint64),
        ("global_cache_bytes", C.c_uint64),
        ("local_memory_bytes", C.c_uint64),
        ("compute_units", C.c_uint32),
        ("max_clock_mhz", C.c_uint32),
        ("svm_capabilities", C.c_uint32),
    ]


@dataclass(frozen=True)
class TraceEvent:
    scope: str
    operation: str
    queued_ns: int
    submit_ns: int
    start_ns: int
    end_ns: int

    @property
    def duration_ns(self) -> int:
        return self.end_ns - self.start_ns

    @property
    def queue_delay_ns(self) -> int:
        return self.start_ns - self.queued_ns


def default_library_path() -> Path:
    return Path(__file__).resolve().parent / "lib" / LIB_NAME


def runtime_paths() -> tuple[Path, None]:
    """(library, kernel source). The second element is always None: kernels
    are compiled ahead of time. ``VLLM_NVFP4_CUDA_LIB`` overrides the library
    path (the lab's ``VLLM_NVFP4_OPENCL_DLL``, runtime.py:64-77)."""
    configured = os.environ.get("VLLM_NVFP4_CUDA_LIB")
    return (Path(configured).resolve() if configured else default_library_path(), None)


def provider_enabled() -> tuple[bool, str | None]:
    """Opt-in gate of the vLLM provider (runtime.py:80-91): requires
    ``VLLM_NVFP4_CUDA=1`` and the built library."""
    if os.environ.get("VLLM_NVFP4_CUDA") != "1":
        return False, "set VLLM_NVFP4_CUDA=1 to opt into the CUDA NVFP4 backend"
    lib, _ = runtime_paths()
    if not lib.is_file():
        return False, f"missing runtime artifact: {lib}"
    return True, None


_SIGNATURES: dict[str, tuple[list, object]] = {
    "nvfp4_last_error": ([], C.c_char_p),
    "nvfp4_runtime_create": ([C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "nvfp4_runtime_destroy": ([C.c_void_p], None),
    "nvfp4_runtime_device_name": ([C.c_void_p], C.c_char_p),
    "nvfp4_runtime_last_profile": ([C.c_void_p, C.POINTER(Profile)], C.c_int),
    "nvfp4_runtime_query_device": ([C.c_void_p, C.POINTER(_DeviceInfo)], C.c_int),
    "nvfp4_runtime_synchronize": ([C.c_void_p], C.c_int),
    "nvfp4_runtime_trace_set_enabled": ([C.c_void_p, C.c_int], C.c_int),
    "nvfp4_runtime_trace_set_scope": ([C.c_void_p, C.c_char_p], C.c_int),
    "nvfp4_runtime_trace_count": ([C.c_void_p], C.c_size_t),
    "nvfp4_runtime_trace_read": ([C.c_void_p, C.c_size_t, C.POINTER(_NativeTraceEvent)], C.c_int),
    "nvfp4_runtime_stream": ([C.c_void_p], C.c_void_p),
    "nvfp4_runtime_sm_count": ([C.c_void_p], C.c_int),
    "nvfp4_buffer_create": ([C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)], C.c_int),
    "nvfp4_buffer_destroy": ([C.c_void_p], None),
    "nvfp4_buffer_upload": ([C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t], C.c_int),
    "nvfp4_buffer_download": ([C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t], C.c_int),
    "nvfp4_buffer_copy_enqueue": ([C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t], C.c_int),
    "nvfp4_buffer_device_pointer": ([C.c_void_p], C.c_void_p),
    "nvfp4_buffer_bytes": ([C.c_void_p], C.c_size_t),
    "nvfp4_add_device_enqueue_f32": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_weighted_accumulate_device_enqueue_f32": (
        [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_int, C.c_int], C.c_int),
    "nvfp4_silu_mul_device_enqueue_f32": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_rmsnorm_device_enqueue_f32": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p], C.c_int),
    "nvfp4_rmsnorm_device_enqueue_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p], C.c_int),
    "nvfp4_bf16_gemv_device_enqueue": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_moe_bank_create": (
        [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int,
         C.POINTER(C.c_void_p)], C.c_int),
    "nvfp4_moe_bank_upload_projection": (
        [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_float], C.c_int),
    "nvfp4_moe_bank_upload_projection_device": (
        [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_float], C.c_int),
    "nvfp4_moe_bank_decode_device_enqueue_f32": ([C.c_void_p, C.c_void_p, C.c_void_p], C.c_int),
    "nvfp4_moe_bank_forward_device_enqueue_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_moe_bank_forward_ptr_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_moe_bank_forward_host_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int], C.c_int),
    "nvfp4_moe_bank_last_routing": (
        [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int)], C.c_int),
    "nvfp4_moe_bank_last_logits": ([C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_int)], C.c_int),
    "nvfp4_moe_bank_set_router_bias": ([C.c_void_p, C.c_void_p, C.c_int], C.c_int),
    "nvfp4_moe_bank_info": (
        [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_size_t)],
        C.c_int),
    "nvfp4_moe_bank_destroy": ([C.c_void_p], None),
    "nvfp4_moe_route_static_scratch": (
        [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
         C.c_void_p], C.c_int),
    "nvfp4_moe_bank_set_prefill_terms": ([C.c_void_p, C.c_int, C.c_int], C.c_int),
    "nvfp4_moe_bank_reserve_prefill": ([C.c_void_p, C.c_int], C.c_int),
    "nvfp4_moe_bank_set_decode_kernels": ([C.c_void_p, C.c_int], C.c_int),
    "nvfp4_moe_bank_set_pre_norm": ([C.c_void_p, C.c_void_p, C.c_float], C.c_int),
    "nvfp4_moe_bank_set_expert_range": ([C.c_void_p, C.c_int, C.c_int, C.c_int], C.c_int),
    "nvfp4_ep_create": ([C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "nvfp4_ep_ipc_handle": ([C.c_void_p, C.c_void_p], C.c_int),
    "nvfp4_ep_open_peers": ([C.c_void_p, C.c_void_p], C.c_int),
    "nvfp4_ep_destroy": ([C.c_void_p], None),
    "nvfp4_moe_bank_forward_ep_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_moe_finalize_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "nvfp4_rmsnorm_ptr_bf16": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_void_p], C.c_int),
    "nvfp4_matrix_upload": (
        [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_float,
         C.POINTER(C.c_void_p)], C.c_int),
    "nvfp4_matrix_destroy": ([C.c_void_p], None),
    "nvfp4_linear_f32": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int], C.c_int),
    "nvfp4_linear_device_f32": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int], C.c_int),
    "nvfp4_linear_device_enqueue_f32": (
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int], C.c_int),
    "nvfp4_linear_ptr_f32": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
    "nvfp4_quantize_rows_enqueue": (
        [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p],
        C.c_int),
}


def load_library(path: Path | None = None) -> C.CDLL:
    """Load the CUDA library and declare every entry point's signature."""
    lib_path = path or runtime_paths()[0]
    if not Path(lib_path).is_file():
        raise RuntimeError(
            f"{LIB_NAME} not found at {lib_path}; build it with x2-nvfp4-lab_b200/build.py"
        )
    lib = C.CDLL(str(lib_path))
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


# cudaStreamLegacy: the legacy default stream as an explicit handle.
CUDA_STREAM_LEGACY = 1


def _current_cuda_device() -> int | None:
    """The calling thread's CUDA device, the one a runtime created on this
    thread binds; None when torch has no CUDA."""
    try:
        import torch
    except ImportError:
        return None
    return torch.cuda.current_device() if torch.cuda.is_available() else None


def _stream_handle(stream) -> C.c_void_p:
    """Handle of a torch.cuda.Stream for the C ABI. torch's default stream has
    handle 0, which the ABI would read as "the runtime's own stream" (not
    ordered with torch's work), so it is passed as cudaStreamLegacy."""
    return C.c_void_p(stream.cuda_stream or CUDA_STREAM_LEGACY)


def _ptr(array: np.ndarray) -> C.c_void_p:
    return C.c_void_p(array.ctypes.data)


def _tensor_ptr(tensor) -> C.c_void_p:
    return C.c_void_p(tensor.data_ptr())


_BF16 = None


def _torch_bf16():
    """torch.bfloat16, imported on first use (the numpy-only paths never import torch)."""
    global _BF16
    if _BF16 is None:
        import torch

        _BF16 = torch.bfloat16
    return _BF16


class DeviceBuffer:
    def __init__(self, runtime: "Runtime", handle: C.c_void_p, bytes_: int):
        self.runtime = runtime
        self.handle = handle
        self.bytes = bytes_

    @property
    def device_pointer(self) -> int:
        return int(self.runtime.lib.nvfp4_buffer_device_pointer(self.handle) or 0)

    def upload(self, array: np.ndarray, offset: int = 0) -> None:
        if not array.flags.c_contiguous:
            raise ValueError("upload array must be contiguous")
        self.runtime._check(
            self.runtime.lib.nvfp4_buffer_upload(self.handle, offset, _ptr(array), array.nbytes),
            "buffer_upload",
        )

    def download(self, shape: tuple[int, ...], dtype: np.dtype | None = None) -> np.ndarray:
        if dtype is None:
            dtype = np.dtype(np.float32)
        output = np.empty(shape, dtype=dtype)
        if output.nbytes > self.bytes:
            raise ValueError("download shape exceeds device-buffer capacity")
        self.runtime._check(
            self.runtime.lib.nvfp4_buffer_download(self.handle, 0, _ptr(output), output.nbytes),
            "buffer_download",
        )
        return output

    def close(self) -> None:
        if self.handle:
            self.runtime.lib.nvfp4_buffer_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


@dataclass
class Routing:
    """additive: routing record of the most recent bank call."""

    ids: np.ndarray       # int32 [T, 9], slot 8 = shared expert id
    weights: np.ndarray   # float32 [T, 9], slot 8 = sigmoid(shared logit)
    counts: np.ndarray    # int32 [experts]
    perm: np.ndarray      # int32 [T*8]


class EpContext:
    """additive: one rank's buffers for the fused expert-parallel combine
    (nvfp4_ep_*). Exchange ``ipc_handle()`` with every rank, then call
    ``open_peers(handles_in_rank_order)``."""

    HANDLE_BYTES = 64

    def __init__(self, runtime: "Runtime", rank: int, world: int, max_tokens: int, hidden: int):
        self.runtime = runtime
        self.rank, self.world, self.max_tokens, self.hidden = rank, world, max_tokens, hidden
        self.handle = C.c_void_p()
        runtime._check(runtime.lib.nvfp4_ep_create(runtime.handle, rank, world, max_tokens, hidden,
                                                   C.byref(self.handle)), "nvfp4_ep_create")

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(self.HANDLE_BYTES)
        self.runtime._check(self.runtime.lib.nvfp4_ep_ipc_handle(self.handle, buf), "nvfp4_ep_ipc_handle")
        return buf.raw

    def open_peers(self, handles: list[bytes]) -> None:
        if len(handles) != self.world or any(len(h) != self.HANDLE_BYTES for h in handles):
            raise ValueError("one handle per rank expected")
        blob = C.create_string_buffer(b"".join(handles), self.HANDLE_BYTES * self.world)
        self.runtime._check(self.runtime.lib.nvfp4_ep_open_peers(self.handle, blob), "nvfp4_ep_open_peers")

    def close(self) -> None:
        if self.handle:
            self.runtime.lib.nvfp4_ep_destroy(self.handle)
            self.handle = C.c_void_p()


class NativeMatrix:
    """A dense NVFP4 weight matrix resident on the device (runtime.py:94-115)."""

    def __init__(self, runtime: "Runtime", handle: C.c_void_p, rows: int, cols: int):
        self.runtime = runtime
        self.handle = handle
        self.rows = rows
        self.cols = cols
        self.shared_svm = False  # the lab's Adreno SVM placement has no counterpart here
        self.device = _current_cuda_device()  # the runtime's device at upload (None without torch CUDA)

    def close(self) -> None:
        if self.handle:
            self.runtime.lib.nvfp4_matrix_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


KERNEL_SCALAR, KERNEL_SUBGROUP, KERNEL_TILED, KERNEL_ROW_TILED = 0, 1, 2, 3


class MoeBank:
    def __init__(self, runtime: "Runtime", handle: C.c_void_p, experts: int, hidden: int, intermediate: int):
        self.runtime = runtime
        self.handle = handle
        self.experts = experts
        self.hidden = hidden
        self.intermediate = intermediate

    def _shape(self, projection: int) -> tuple[int, int]:
        return (self.intermediate, self.hidden) if projection < 2 else (self.hidden, self.intermediate)

    def upload_projection(
        self,
        expert: int,
        projection: int,
        packed: np.ndarray,
        scales: np.ndarray,
        checkpoint_global_scale: float,
    ) -> None:
        """Same checks and meaning as the lab (runtime.py:321-358):
        ``checkpoint_global_scale`` is the divisor 1/weight_scale_2."""
        if projection not in (0, 1, 2):
            raise ValueError("projection must be 0=gate, 1=up, or 2=down")
        rows, cols = self._shape(projection)
        if (
            not 0 <= expert <= self.experts
            or packed.shape != (rows, cols // 2)
            or scales.shape != (rows, cols // 16)
            or packed.dtype != np.uint8
            or scales.dtype != np.uint8
            or not packed.flags.c_contiguous
            or not scales.flags.c_contiguous
        ):
            raise ValueError("invalid contiguous uint8 MoE projection")
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_upload_projection(
                self.handle, expert, projection, _ptr(packed), packed.nbytes, _ptr(scales), scales.nbytes,
                checkpoint_global_scale,
            ),
            "nvfp4_moe_bank_upload_projection",
        )

    def upload_expert(self, expert: int, projections: list[tuple[np.ndarray, np.ndarray, float]]) -> None:
        if len(projections) != 3:
            raise ValueError("an MoE expert requires gate, up, and down projections")
        for projection, values in enumerate(projections):
            self.upload_projection(expert, projection, *values)

    def upload_projection_tensor(self, expert: int, projection: int, packed, scales,
                                 checkpoint_global_scale: float) -> None:
        """additive: upload from contiguous CUDA uint8 tensors (enqueued on the
        runtime stream; keep the tensors alive until the next synchronize)."""
        rows, cols = self._shape(projection)
        if (
            tuple(packed.shape) != (rows, cols // 2)
            or tuple(scales.shape) != (rows, cols // 16)
            or not packed.is_cuda
            or not scales.is_cuda
            or not packed.is_contiguous()
            or not scales.is_contiguous()
        ):
            raise ValueError("invalid contiguous CUDA uint8 MoE projection")
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_upload_projection_device(
                self.handle, expert, projection, _tensor_ptr(packed), packed.numel(), _tensor_ptr(scales),
                scales.numel(), float(checkpoint_global_scale),
            ),
            "nvfp4_moe_bank_upload_projection_device",
        )

    def decode_device(self, x: DeviceBuffer, out: DeviceBuffer) -> DeviceBuffer:
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_decode_device_enqueue_f32(self.handle, x.handle, out.handle),
            "nvfp4_moe_bank_decode_device_enqueue_f32",
        )
        return out

    def forward_device(self, x: DeviceBuffer, tokens: int, out: DeviceBuffer,
                       residual: DeviceBuffer | None = None) -> DeviceBuffer:
        """additive: BF16 [tokens, hidden] buffers; residual added when given."""
        flags = NVFP4_MOE_ADD_RESIDUAL if residual is not None else 0
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_forward_device_enqueue_bf16(
                self.handle, x.handle, residual.handle if residual is not None else None, tokens, flags,
                out.handle,
            ),
            "nvfp4_moe_bank_forward_device_enqueue_bf16",
        )
        return out

    def forward_host(self, x, residual=None, out=None, pre_norm: bool = False):
        """additive: one end-to-end call on host memory (nvfp4_moe_bank_forward_host_bf16):
        x, residual and out are CPU BF16 torch tensors [tokens, hidden] (pinned
        for asynchronous copies) or uint16/int16 numpy arrays of BF16 bits.
        Returns out once the result is in it."""
        # Called once per layer call on the end-to-end path: each check is one
        # attribute read, and pointers go to ctypes as plain integers.
        def host_ptr(a, name):
            if a is None:
                return None, None
            if isinstance(a, np.ndarray):
                if a.dtype not in (np.uint16, np.int16) or a.ndim != 2 or a.shape[1] != self.hidden \
                        or not a.flags.c_contiguous:
                    raise ValueError(f"{name} must be contiguous BF16 bits [tokens, hidden]")
                return a.ctypes.data, a.shape[0]
            shape = a.shape
            if a.dtype is not _torch_bf16() or len(shape) != 2 or shape[1] != self.hidden or a.is_cuda \
                    or not a.is_contiguous():
                raise ValueError(f"{name} must be a contiguous CPU bfloat16 tensor [tokens, hidden]")
            return a.data_ptr(), shape[0]

        xp, T = host_ptr(x, "x")
        if out is None:
            if isinstance(x, np.ndarray):
                out = np.empty_like(x)
            else:
                import torch

                out = torch.empty_like(x, pin_memory=x.is_pinned())
        op, To = host_ptr(out, "out")
        rp, Tr = host_ptr(residual, "residual")
        if To != T or (residual is not None and Tr != T):
            raise ValueError("x, residual and out must have the same number of tokens")
        flags = (NVFP4_MOE_ADD_RESIDUAL if residual is not None else 0) | (NVFP4_MOE_PRE_NORM if pre_norm else 0)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_forward_host_bf16(self.handle, xp, rp, op, T, flags),
            "nvfp4_moe_bank_forward_host_bf16")
        return out

    def forward(self, x, residual=None, out=None, stream=None, pre_norm: bool = False):
        """additive: torch BF16 [tokens, hidden] CUDA tensors; enqueued on
        ``stream`` (a torch.cuda.Stream) or torch's current stream. With
        ``pre_norm`` x is first normalised with the weight of ``set_pre_norm``
        (``out`` must then not share memory with x or the residual)."""
        import torch

        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("x must be a CUDA bfloat16 tensor [tokens, hidden]")
        x = x.contiguous()
        if out is None:
            out = torch.empty_like(x)
        flags = NVFP4_MOE_PRE_NORM if pre_norm else 0
        if residual is not None:
            if residual.shape != x.shape or residual.dtype != torch.bfloat16 or not residual.is_cuda:
                raise ValueError("residual must match x")
            residual = residual.contiguous()
            flags |= NVFP4_MOE_ADD_RESIDUAL
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_forward_ptr_bf16(
                self.handle, _tensor_ptr(x), _tensor_ptr(residual) if residual is not None else None,
                _tensor_ptr(out), x.shape[0], flags, _stream_handle(s),
            ),
            "nvfp4_moe_bank_forward_ptr_bf16",
        )
        return out

    def forward_partial(self, x, out=None, residual=None, stream=None):
        """additive (expert parallelism): FP32 [tokens, hidden] partial sum of
        this bank's expert range (set_expert_range), plus ``residual`` when
        given. Summing the partials of ranks that cover every expert once
        gives the layer output before its BF16 rounding."""
        import torch

        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("x must be a CUDA bfloat16 tensor [tokens, hidden]")
        x = x.contiguous()
        if out is None:
            out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        if out.dtype != torch.float32 or out.shape != x.shape or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 tensor shaped like x")
        flags = NVFP4_MOE_PARTIAL_F32
        if residual is not None:
            if residual.shape != x.shape or residual.dtype != torch.bfloat16 or not residual.is_cuda:
                raise ValueError("residual must match x")
            residual = residual.contiguous()
            flags |= NVFP4_MOE_ADD_RESIDUAL
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_forward_ptr_bf16(
                self.handle, _tensor_ptr(x), _tensor_ptr(residual) if residual is not None else None,
                _tensor_ptr(out), x.shape[0], flags, _stream_handle(s),
            ),
            "nvfp4_moe_bank_forward_ptr_bf16",
        )
        return out

    def forward_ep(self, ep: "EpContext", x, residual=None, out=None, stream=None):
        """additive (expert parallelism, reduction fused into the combine over
        NVLink peer memory): the whole layer's BF16 output on every rank; call
        on every rank with the same x (at most ep.max_tokens tokens)."""
        import torch

        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("x must be a CUDA bfloat16 tensor [tokens, hidden]")
        x = x.contiguous()
        if out is None:
            out = torch.empty_like(x)
        flags = 0
        if residual is not None:
            if residual.shape != x.shape or residual.dtype != torch.bfloat16 or not residual.is_cuda:
                raise ValueError("residual must match x")
            residual = residual.contiguous()
            flags = NVFP4_MOE_ADD_RESIDUAL
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_forward_ep_bf16(
                self.handle, ep.handle, _tensor_ptr(x), _tensor_ptr(residual) if residual is not None else None,
                _tensor_ptr(out), x.shape[0], flags, _stream_handle(s)),
            "nvfp4_moe_bank_forward_ep_bf16")
        return out

    def set_expert_range(self, first: int, count: int, shared_here: bool) -> None:
        """additive (expert parallelism): compute routed experts [first, first + count)
        and the shared expert when ``shared_here``."""
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_set_expert_range(self.handle, first, count, 1 if shared_here else 0),
            "nvfp4_moe_bank_set_expert_range")

    def last_routing(self, max_tokens: int) -> Routing:
        """additive: routing of the most recent call (synchronises)."""
        ids = np.zeros((max_tokens, 9), dtype=np.int32)
        weights = np.zeros((max_tokens, 9), dtype=np.float32)
        counts = np.zeros(self.experts, dtype=np.int32)
        perm = np.zeros(max_tokens * 8, dtype=np.int32)
        tokens = C.c_int(0)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_last_routing(
                self.handle, max_tokens, _ptr(ids), _ptr(weights), _ptr(counts), _ptr(perm), C.byref(tokens)
            ),
            "nvfp4_moe_bank_last_routing",
        )
        t = min(tokens.value, max_tokens)
        return Routing(ids[:t], weights[:t], counts, perm[: t * 8])

    def last_logits(self, max_tokens: int) -> np.ndarray:
        logits = np.zeros((max_tokens, self.experts + 1), dtype=np.float32)
        tokens = C.c_int(0)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_last_logits(self.handle, max_tokens, _ptr(logits), C.byref(tokens)),
            "nvfp4_moe_bank_last_logits",
        )
        return logits[: min(tokens.value, max_tokens)]

    def set_router_bias(self, bias: np.ndarray | None) -> None:
        """additive: FP32 per-expert router logit bias (None clears it)."""
        if bias is None:
            self.runtime._check(self.runtime.lib.nvfp4_moe_bank_set_router_bias(self.handle, None, 0),
                                "nvfp4_moe_bank_set_router_bias")
            return
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        if bias.shape != (self.experts,):
            raise ValueError("router bias must be float32 [experts]")
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_set_router_bias(self.handle, _ptr(bias), self.experts),
            "nvfp4_moe_bank_set_router_bias",
        )

    def set_prefill_terms(self, x_terms: int, act_terms: int) -> None:
        """additive: NVFP4 activation terms of the prefill path (1..4 each)."""
        self.runtime._check(self.runtime.lib.nvfp4_moe_bank_set_prefill_terms(self.handle, x_terms, act_terms),
                            "nvfp4_moe_bank_set_prefill_terms")

    def set_pre_norm(self, weight=None, epsilon: float = 1e-6) -> None:
        """additive: the RMSNorm of ``forward(..., pre_norm=True)``: a CUDA
        bfloat16 tensor [hidden] (copied into the bank) or None for ones."""
        import torch

        ptr = None
        if weight is not None:
            if weight.dtype != torch.bfloat16 or not weight.is_cuda or weight.numel() != self.hidden:
                raise ValueError("weight must be a CUDA bfloat16 tensor with hidden entries")
            weight = weight.contiguous()
            ptr = _tensor_ptr(weight)
        self.runtime._check(self.runtime.lib.nvfp4_moe_bank_set_pre_norm(self.handle, ptr, float(epsilon)),
                            "nvfp4_moe_bank_set_pre_norm")

    def set_decode_kernels(self, kernels: str) -> None:
        """additive: decode expert-GEMV variant, "tensor_core" (default), "in_register" or
        "fused_token" (tensor-core, one-token calls as one persistent kernel)."""
        code = {"tensor_core": NVFP4_DECODE_KERNELS_TENSOR_CORE, "in_register": NVFP4_DECODE_KERNELS_IN_REGISTER,
                "fused_token": NVFP4_DECODE_KERNELS_FUSED_TOKEN}
        if kernels not in code:
            raise ValueError(f"unknown decode kernels {kernels!r}")
        self.runtime._check(self.runtime.lib.nvfp4_moe_bank_set_decode_kernels(self.handle, code[kernels]),
                            "nvfp4_moe_bank_set_decode_kernels")

    def reserve_prefill(self, max_tokens: int) -> None:
        """additive: allocate prefill working memory for calls of up to max_tokens tokens."""
        self.runtime._check(self.runtime.lib.nvfp4_moe_bank_reserve_prefill(self.handle, max_tokens),
                            "nvfp4_moe_bank_reserve_prefill")

    @property
    def resident_bytes(self) -> int:
        size = C.c_size_t(0)
        self.runtime._check(
            self.runtime.lib.nvfp4_moe_bank_info(self.handle, None, None, None, C.byref(size)),
            "nvfp4_moe_bank_info",
        )
        return int(size.value)

    def close(self) -> None:
        if self.handle:
            self.runtime.lib.nvfp4_moe_bank_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class Runtime:
    def __init__(self, lib_path: Path | None = None, kernel_path: Path | None = None):
        self.lib = load_library(lib_path)
        self.handle = C.c_void_p()
        self._check(
            self.lib.nvfp4_runtime_create(
                str(kernel_path).encode() if kernel_path else None, C.byref(self.handle)
            ),
            "runtime_create",
        )

    def _check(self, status: int, operation: str) -> None:
        if status:
            error = (self.lib.nvfp4_last_error() or b"").decode(errors="replace")
            raise RuntimeError(f"{operation} failed ({status}): {error}")

    @property
    def device_name(self) -> str:
        value = self.lib.nvfp4_runtime_device_name(self.handle)
        return value.decode(errors="replace") if value else "unknown"

    @property
    def stream_handle(self) -> int:
        """additive: the runtime's cudaStream_t as an integer."""
        return int(self.lib.nvfp4_runtime_stream(self.handle) or 0)

    @property
    def sm_count(self) -> int:
        return int(self.lib.nvfp4_runtime_sm_count(self.handle))

    def query_device(self) -> dict:
        info = _DeviceInfo()
        self._check(self.lib.nvfp4_runtime_query_device(self.handle, C.byref(info)), "runtime_query_device")
        return {
            "platform_name": info.platform_name.decode(),
            "device_name": info.device_name.decode(),
            "device_version": info.device_version.decode(),
            "driver_version": info.driver_version.decode(),
            "global_memory_bytes": int(info.global_memory_bytes),
            "global_cache_bytes": int(info.global_cache_bytes),
            "compute_units": int(info.compute_units),
            "max_clock_mhz": int(info.max_clock_mhz),
        }

    def last_profile(self) -> Profile:
        profile = Profile()
        self._check(self.lib.nvfp4_runtime_last_profile(self.handle, C.byref(profile)), "runtime_last_profile")
        return profile

    def synchronize(self) -> Profile:
        self._check(self.lib.nvfp4_runtime_synchronize(self.handle), "runtime_synchronize")
        return self.last_profile()

    def set_trace_enabled(self, enabled: bool) -> None:
        self._check(self.lib.nvfp4_runtime_trace_set_enabled(self.handle, int(enabled)), "runtime_trace_set_enabled")

    def set_trace_scope(self, scope: str) -> None:
        encoded = scope.encode("utf-8")
        if len(encoded) >= 96:
            raise ValueError("trace scope must be shorter than 96 UTF-8 bytes")
        self._check(self.lib.nvfp4_runtime_trace_set_scope(self.handle, encoded), "runtime_trace_set_scope")

    def trace_events(self) -> list[TraceEvent]:
        count = int(self.lib.nvfp4_runtime_trace_count(self.handle))
        events = []
        for index in range(count):
            native = _NativeTraceEvent()
            self._check(self.lib.nvfp4_runtime_trace_read(self.handle, index, C.byref(native)), "runtime_trace_read")
            events.append(
                TraceEvent(
                    scope=bytes(native.scope).split(b"\0", 1)[0].decode(),
                    operation=bytes(native.operation).split(b"\0", 1)[0].decode(),
                    queued_ns=int(native.queued_ns),
                    submit_ns=int(native.submit_ns),
                    start_ns=int(native.start_ns),
                    end_ns=int(native.end_ns),
                )
            )
        return events

    def create_buffer(self, bytes_: int) -> DeviceBuffer:
        if bytes_ <= 0:
            raise ValueError("device-buffer size must be positive")
        handle = C.c_void_p()
        self._check(self.lib.nvfp4_buffer_create(self.handle, bytes_, C.byref(handle)), "buffer_create")
        return DeviceBuffer(self, handle, bytes_)

    def upload_buffer(self, array: np.ndarray) -> DeviceBuffer:
        buffer = self.create_buffer(array.nbytes)
        try:
            buffer.upload(array)
        except Exception:
            buffer.close()
            raise
        return buffer

    def copy_buffer_device(self, source: DeviceBuffer, destination: DeviceBuffer, bytes_: int,
                           source_offset: int = 0, destination_offset: int = 0) -> None:
        if bytes_ <= 0 or source_offset < 0 or destination_offset < 0:
            raise ValueError("buffer copy ranges must be nonnegative and nonempty")
        self._check(
            self.lib.nvfp4_buffer_copy_enqueue(source.handle, source_offset, destination.handle,
                                               destination_offset, bytes_),
            "buffer_copy_enqueue",
        )

    def create_moe_bank(self, router_bf16: np.ndarray, shared_gate_bf16: np.ndarray, intermediate: int) -> MoeBank:
        """Same checks as the lab (runtime.py:986-1024): router BF16 bits
        [8..256, hidden], shared gate BF16 bits [hidden]."""
        if (
            router_bf16.ndim != 2
            or router_bf16.dtype != np.uint16
            or not router_bf16.flags.c_contiguous
            or router_bf16.shape[0] < 8
            or router_bf16.shape[0] > 256
            or intermediate <= 0
            or intermediate % 16 != 0
        ):
            raise ValueError("router must be contiguous BF16 bits [8..256, hidden]")
        shared_gate_bf16 = np.ascontiguousarray(shared_gate_bf16.reshape(-1))
        if shared_gate_bf16.dtype != np.uint16 or shared_gate_bf16.size != router_bf16.shape[1]:
            raise ValueError("shared gate must be BF16 bits [hidden]")
        experts, hidden = router_bf16.shape
        handle = C.c_void_p()
        self._check(
            self.lib.nvfp4_moe_bank_create(
                self.handle, _ptr(router_bf16), router_bf16.nbytes, _ptr(shared_gate_bf16),
                shared_gate_bf16.nbytes, experts, hidden, intermediate, C.byref(handle),
            ),
            "nvfp4_moe_bank_create",
        )
        return MoeBank(self, handle, experts, hidden, intermediate)

    def add_device(self, a: DeviceBuffer, b: DeviceBuffer, elements: int, out: DeviceBuffer) -> DeviceBuffer:
        self._check(self.lib.nvfp4_add_device_enqueue_f32(self.handle, a.handle, b.handle, elements, out.handle),
                    "add_device_enqueue_f32")
        return out

    def silu_mul_device(self, gate: DeviceBuffer, up: DeviceBuffer, elements: int, out: DeviceBuffer) -> DeviceBuffer:
        self._check(
            self.lib.nvfp4_silu_mul_device_enqueue_f32(self.handle, gate.handle, up.handle, elements, out.handle),
            "silu_mul_device_enqueue_f32",
        )
        return out

    def weighted_accumulate_device(self, source: DeviceBuffer, scale: float, out: DeviceBuffer, elements: int,
                                   *, reset: bool = False) -> DeviceBuffer:
        self._check(
            self.lib.nvfp4_weighted_accumulate_device_enqueue_f32(self.handle, source.handle, scale, out.handle,
                                                                  elements, int(reset)),
            "weighted_accumulate_device_enqueue_f32",
        )
        return out

    def rmsnorm_device(self, x: DeviceBuffer, weight: DeviceBuffer, rows: int, cols: int, epsilon: float,
                       out: DeviceBuffer) -> DeviceBuffer:
        self._check(
            self.lib.nvfp4_rmsnorm_device_enqueue_f32(self.handle, x.handle, weight.handle, rows, cols, epsilon,
                                                      out.handle),
            "rmsnorm_device_enqueue_f32",
        )
        return out

    def rmsnorm_device_bf16(self, x: DeviceBuffer, weight: DeviceBuffer, rows: int, cols: int, epsilon: float,
                            out: DeviceBuffer) -> DeviceBuffer:
        """additive: BF16 RMSNorm."""
        self._check(
            self.lib.nvfp4_rmsnorm_device_enqueue_bf16(self.handle, x.handle, weight.handle, rows, cols, epsilon,
                                                       out.handle),
            "rmsnorm_device_enqueue_bf16",
        )
        return out

    def bf16_gemv_device(self, weights: DeviceBuffer, x: DeviceBuffer, rows: int, cols: int,
                         out: DeviceBuffer) -> DeviceBuffer:
        self._check(
            self.lib.nvfp4_bf16_gemv_device_enqueue(self.handle, weights.handle, x.handle, rows, cols, out.handle),
            "bf16_gemv_device_enqueue",
        )
        return out

    def finalize_bf16(self, sum_f32, residual=None, out=None, stream=None):
        """additive (expert parallelism): BF16(sum_f32 + residual) for torch CUDA
        tensors [tokens, hidden] (sum FP32, residual BF16 or None)."""
        import torch

        if sum_f32.dtype != torch.float32 or not sum_f32.is_cuda or sum_f32.dim() != 2:
            raise ValueError("sum_f32 must be a CUDA float32 tensor [tokens, hidden]")
        sum_f32 = sum_f32.contiguous()
        if out is None:
            out = torch.empty(sum_f32.shape, dtype=torch.bfloat16, device=sum_f32.device)
        if residual is not None:
            if residual.shape != sum_f32.shape or residual.dtype != torch.bfloat16:
                raise ValueError("residual must be bfloat16 shaped like sum_f32")
            residual = residual.contiguous()
        s = stream if stream is not None else torch.cuda.current_stream(sum_f32.device)
        self._check(
            self.lib.nvfp4_moe_finalize_bf16(
                self.handle, _tensor_ptr(sum_f32), _tensor_ptr(residual) if residual is not None else None,
                _tensor_ptr(out), sum_f32.shape[0], sum_f32.shape[1], _stream_handle(s)),
            "nvfp4_moe_finalize_bf16")
        return out

    def rmsnorm_bf16(self, x, weight, epsilon: float = 1e-6, out=None, stream=None):
        """additive: BF16 RMSNorm of the rows of a CUDA bfloat16 tensor [rows, cols]
        with a bfloat16 weight [cols] (the layer stack's pre-norm), enqueued on
        ``stream`` (None: torch's current stream)."""
        import torch

        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2:
            raise ValueError("x must be a CUDA bfloat16 tensor [rows, cols]")
        if weight.dtype != torch.bfloat16 or weight.numel() != x.shape[1]:
            raise ValueError("weight must be bfloat16 with one entry per column")
        x = x.contiguous()
        weight = weight.contiguous()
        if out is None:
            out = torch.empty_like(x)
        elif out.shape != x.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bfloat16 tensor shaped like x")
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self._check(
            self.lib.nvfp4_rmsnorm_ptr_bf16(self.handle, _tensor_ptr(x), _tensor_ptr(weight), x.shape[0], x.shape[1],
                                            float(epsilon), _tensor_ptr(out), _stream_handle(s)),
            "nvfp4_rmsnorm_ptr_bf16")
        return out

    def upload(self, packed: np.ndarray, scales: np.ndarray, checkpoint_global_scale: float, *,
               shared_svm: bool | None = None) -> NativeMatrix:
        """A dense NVFP4 matrix from the compressed-tensors representation
        (runtime.py:927-990): packed uint8 [rows, cols/2], scales E4M3 bytes
        [rows, cols/16], and the divisor of the dequantised weights. The lab's
        ``shared_svm`` placement is an Adreno memory mode; device memory is
        used whatever it says."""
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        scales = np.ascontiguousarray(scales).view(np.uint8)
        if packed.ndim != 2:
            raise ValueError("packed must be uint8 [rows, cols/2]")
        handle = C.c_void_p()
        self._check(
            self.lib.nvfp4_matrix_upload(self.handle, _ptr(packed), packed.nbytes, _ptr(scales), scales.nbytes,
                                         packed.shape[0], packed.shape[1] * 2, float(checkpoint_global_scale),
                                         C.byref(handle)),
            "matrix_upload",
        )
        return NativeMatrix(self, handle, packed.shape[0], packed.shape[1] * 2)

    def linear(self, matrix: NativeMatrix, x: np.ndarray, kernel_kind: int | None = None) -> np.ndarray:
        """Synchronous linear on host arrays (runtime.py:1095-1125): x float32
        [vectors, cols] -> float32 [vectors, rows]."""
        if x.ndim != 2 or x.shape[1] != matrix.cols or x.dtype != np.float32:
            raise ValueError("x must be contiguous float32 [vectors, cols]")
        x = np.ascontiguousarray(x)
        out = np.empty((x.shape[0], matrix.rows), dtype=np.float32)
        kind = kernel_kind if kernel_kind is not None else (
            KERNEL_TILED if x.shape[0] > 1 else (KERNEL_ROW_TILED if matrix.rows <= 1024 else KERNEL_SUBGROUP))
        self._check(
            self.lib.nvfp4_linear_f32(self.handle, matrix.handle, _ptr(x), x.shape[0], _ptr(out), int(kind)),
            "linear",
        )
        return out

    def linear_device(self, matrix: NativeMatrix, x: DeviceBuffer, vectors: int, out: DeviceBuffer,
                      kernel_kind: int = KERNEL_SUBGROUP, enqueue: bool = False) -> DeviceBuffer:
        """Linear on device buffers: waits for the kernel, or only enqueues it
        on the runtime stream with ``enqueue``."""
        fn = self.lib.nvfp4_linear_device_enqueue_f32 if enqueue else self.lib.nvfp4_linear_device_f32
        self._check(fn(self.handle, matrix.handle, x.handle, vectors, out.handle, int(kernel_kind)),
                    "linear_device_enqueue" if enqueue else "linear_device")
        return out

    def linear_tensor(self, matrix: NativeMatrix, x, out=None, stream=None):
        """additive: the linear on a CUDA float32 tensor [..., cols], enqueued on
        ``stream`` (None: torch's current stream); returns float32 [..., rows]."""
        import torch

        if x.dtype != torch.float32 or not x.is_cuda or x.shape[-1] != matrix.cols:
            raise ValueError("x must be a CUDA float32 tensor [..., cols]")
        home = getattr(matrix, "device", None)
        for name, t in (("x", x), ("out", out)):
            if t is not None and home is not None and t.device.index != home:
                raise ValueError(f"{name} is on {t.device} but the matrix is resident on cuda:{home}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, matrix.cols).contiguous()
        if out is None:
            out = torch.empty(*lead, matrix.rows, dtype=torch.float32, device=x.device)
        elif out.dtype != torch.float32 or tuple(out.shape) != (*lead, matrix.rows) or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 tensor [..., rows]")
        if x2.shape[0] == 0:
            return out
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self._check(
            self.lib.nvfp4_linear_ptr_f32(self.handle, matrix.handle, _tensor_ptr(x2), x2.shape[0],
                                          _tensor_ptr(out), _stream_handle(s)),
            "nvfp4_linear_ptr_f32",
        )
        return out

    def quantize_rows(self, x, terms: int):
        """additive: split BF16/FP16 rows [rows, cols] (a CUDA tensor) into
        `terms` NVFP4 terms on torch's current stream. Returns (codes uint8
        [terms, rows, cols/2], scale words int32 [terms, rows, cols/64], row
        scales float32 [rows])."""
        import torch

        if x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float16) or not x.is_cuda:
            raise ValueError("quantize_rows expects a 2D BF16 or FP16 CUDA tensor")
        x = x.contiguous()
        rows, cols = x.shape
        codes = torch.empty(terms, rows, cols // 2, dtype=torch.uint8, device=x.device)
        words = torch.empty(terms, rows, cols // 64, dtype=torch.int32, device=x.device)
        g = torch.empty(rows, dtype=torch.float32, device=x.device)
        stream = torch.cuda.current_stream(x.device)
        self._check(
            self.lib.nvfp4_quantize_rows_enqueue(
                _tensor_ptr(x), 1 if x.dtype == torch.float16 else 0, rows, cols, terms, _tensor_ptr(codes),
                _tensor_ptr(words), _tensor_ptr(g), _stream_handle(stream)),
            "nvfp4_quantize_rows_enqueue",
        )
        return codes, words, g

    def close(self) -> None:
        if self.handle:
            self.lib.nvfp4_runtime_destroy(self.handle)
            self.handle = C.c_void_p()


_runtime: Runtime | None = None
_runtime_lock = threading.Lock()


def get_runtime() -> Runtime:
    """Process-wide runtime (runtime.py:1964-1976). Raises when the provider
    is not enabled; there is no fallback."""
    global _runtime
    with _runtime_lock:
        if _runtime is None:
            enabled, reason = provider_enabled()
            if not enabled:
                raise RuntimeError(reason)
            _runtime = Runtime(*runtime_paths())
        return _runtime
