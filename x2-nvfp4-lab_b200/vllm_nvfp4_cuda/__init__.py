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
    """Register the provider in every vLLM process, idempotently. Registers
    the ``nvfp4_moe::forward`` torch custom op used by model code to call a
    resident bank."""
    global _registered
    if _registered:
        return
    from . import ops  # noqa: F401  (defines the custom op on import)

    _registered = True


__all__ = [
    "DeviceBuffer",
    "MoeBank",
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
