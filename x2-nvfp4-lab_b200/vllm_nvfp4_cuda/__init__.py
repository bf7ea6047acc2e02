"""B200 (sm_100a) NVFP4 mixture-of-experts bank behind the lab's runtime API.

Drop-in for the MoE-bank path of hotschmoe/x2-nvfp4-lab's
``vllm_nvfp4_opencl`` package: ``Runtime``, ``MoeBank``, ``DeviceBuffer`` and
``get_runtime`` keep the lab's names and semantics, backed by
``lib/libnvfp4_moe_cuda.so``. ``register()`` is the ``vllm.general_plugins``
entry point (the lab's ``vllm_nvfp4_opencl:register``, __init__.py:8-29).
"""

from __future__ import annotations

from .runtime import (  # noqa: F401
    DeviceBuffer,
    MoeBank,
    NativeMatrix,
    Profile,
    Routing,
    Runtime,
    TraceEvent,
    get_runtime,
    load_library,
    provider_enabled,
    runtime_paths,
)

_registered = False


def register() -> None:
    """Register the provider in every vLLM process, idempotently: the
    ``nvfp4_moe::forward`` torch custom op used by model code to call a
    resident bank and, when vLLM is installed, the dense NVFP4 linear provider
    (``CudaNvFp4LinearKernel``) for the CUDA platform (the lab registers its
    OpenCL provider the same way, __init__.py:8-29)."""
    global _registered
    if _registered:
        return
    from . import ops  # noqa: F401  (defines the custom op on import)

    try:
        from vllm.model_executor.kernels.linear import register_linear_kernel
        from vllm.platforms import PlatformEnum
    except ImportError:
        register_linear_kernel = None
    if register_linear_kernel is not None:
        from .linear import CudaNvFp4LinearKernel

        register_linear_kernel(CudaNvFp4LinearKernel, PlatformEnum.CUDA, kernel_type="nvfp4")
    _registered = True


__all__ = [
    "DeviceBuffer",
    "MoeBank",
    "NativeMatrix",
    "Profile",
    "Routing",
    "Runtime",
    "TraceEvent",
    "get_runtime",
    "load_library",
    "provider_enabled",
    "register",
    "runtime_paths",
]
