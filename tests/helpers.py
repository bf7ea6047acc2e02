"""Shared helpers for the GPU parity tests (host-side only)."""

from __future__ import annotations

import numpy as np

from oracle.nvfp4_oracle import BankHost, bf16_bits_to_f32

# BASELINE output tolerance against the FP32 dequantise-then-matmul oracle.
REL_RMSE_TOL = 2e-3
MAX_ABS_REL_TOL = 1e-2


def upload_bank(runtime, host: BankHost):
    """Create a device bank from a BankHost through the reference upload ABI."""
    bank = runtime.create_moe_bank(np.ascontiguousarray(host.router_bf16), np.ascontiguousarray(host.shared_gate_bf16),
                                   host.intermediate)
    for e in range(host.experts + 1):
        for p in range(3):
            q = host.projections[p][e]
            bank.upload_projection(e, p, np.ascontiguousarray(q.packed), np.ascontiguousarray(q.scales),
                                   q.global_scale)
    if host.router_bias is not None:
        bank.set_router_bias(host.router_bias)
    return bank


def bf16_tensor_to_f32(t) -> np.ndarray:
    import torch

    return t.detach().to(torch.float32).cpu().numpy()


def bits_to_bf16_tensor(bits: np.ndarray, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def f32_of_bits(bits: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(bits)
