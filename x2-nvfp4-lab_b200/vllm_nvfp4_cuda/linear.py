"""vLLM modular NVFP4 linear provider on the CUDA runtime: the counterpart of
the lab's ``OpenCLNvFp4LinearKernel`` (vllm_nvfp4_opencl/linear.py:15-70).

A16 (weights-only NVFP4) linear layers: the layer's checkpoint-native
``weight`` (packed E2M1 pairs), ``weight_scale`` (E4M3 per 16 columns) and
``weight_global_scale`` are uploaded once into a resident ``NativeMatrix``;
``apply_weights`` runs the runtime's dense NVFP4 linear on the activations
(FP32 on the device) and adds the bias. Registered by
``vllm_nvfp4_cuda.register()`` for the CUDA platform.
"""

from __future__ import annotations

import numpy as np
import torch
from vllm.model_executor.kernels.linear.nvfp4 import NvFp4LinearKernel, NvFp4LinearLayerConfig

from .runtime import NativeMatrix, get_runtime, provider_enabled

SM100 = 100


def _require_cuda(x: torch.Tensor) -> None:
    """The provider's device rule (the lab's raises the same way for
    activations on the wrong device, linear.py:57-58)."""
    if x.device.type != "cuda":
        raise RuntimeError("CUDA NVFP4 currently requires CUDA activations")


class CudaNvFp4LinearKernel(NvFp4LinearKernel):
    """Native compressed-tensors W4A16 linear on sm_100a."""

    @classmethod
    def supports_a16(cls) -> bool:
        return True

    @classmethod
    def is_supported(cls, compute_capability: int | None = None) -> tuple[bool, str | None]:
        if compute_capability is not None and compute_capability != SM100:
            return False, f"the CUDA NVFP4 provider is built for sm_100a, not compute capability {compute_capability}"
        return provider_enabled()

    @classmethod
    def can_implement(cls, config: NvFp4LinearLayerConfig) -> tuple[bool, str | None]:
        return True, None

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        """Upload the layer's NVFP4 weight once (linear.py:36-49): the packed
        codes and scale bytes as stored, and the inverse of the layer's
        ``weight_global_scale`` as the matrix's divisor, as the lab passes it."""
        packed = np.ascontiguousarray(layer.weight.detach().cpu().numpy())
        scales = np.ascontiguousarray(layer.weight_scale.detach().cpu().view(torch.uint8).numpy())
        scale_multiplier = float(layer.weight_global_scale.detach().cpu().item())
        layer._cuda_nvfp4_matrix = get_runtime().upload(packed, scales, 1.0 / scale_multiplier)

    def apply_weights(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        """x [..., cols] on the CUDA device -> [..., rows] in x's dtype
        (linear.py:51-68)."""
        matrix: NativeMatrix = layer._cuda_nvfp4_matrix
        _require_cuda(x)
        if x.shape[-1] != matrix.cols:
            raise ValueError(f"input width {x.shape[-1]} does not match matrix width {matrix.cols}")
        x_f32 = x.detach().to(torch.float32)
        out = get_runtime().linear_tensor(matrix, x_f32).to(dtype=x.dtype)
        if bias is not None:
            out = out + bias
        return out


__all__ = ["CudaNvFp4LinearKernel"]
