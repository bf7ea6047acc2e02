"""Seeded synthetic MoE banks with the BASELINE shapes and distributions.

There is no checkpoint on this machine, so benches and GPU tests build banks
from seeds: router and shared gate BF16 ~ N(0, 0.02), expert weights FP32 ~
N(0, 0.02) quantised to NVFP4, activations BF16 ~ N(0, 1), and for skewed
routing a per-expert router bias b_e = 2.0 * log(1 / rank_e^1.2) with ranks a
seeded permutation. Generation and quantisation run in torch on any device
(the GPU for full-size banks).

Quantiser (the lab ships none; this is the BASELINE rule):
  g = amax / (6 * 448)                          per-tensor, FP32
  s_b = E4M3_RNE(blockamax / 6 / g)             per 16 columns, saturating
  code = E2M1_RNE(w / (s_b * g))                ties to the even code
and the ABI divisor is 1/g. Packing puts column 2j in the low nibble.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

# Midpoints between consecutive E2M1 magnitudes {0,.5,1,1.5,2,3,4,6}; a tie
# rounds to the even code, i.e. up at 0.75, 1.75 and 3.5, down elsewhere.
_E2M1_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
_E2M1_TIE_UP = (False, True, False, True, False, True, False)


def e2m1_codes(scaled: torch.Tensor) -> torch.Tensor:
    """float32 tensor -> uint8 E2M1 codes (sign in bit 3)."""
    mag = scaled.abs().clamp(max=6.0)
    code = torch.zeros_like(mag, dtype=torch.uint8)
    for mid, tie_up in zip(_E2M1_MIDPOINTS, _E2M1_TIE_UP):
        step = (mag > mid) | ((mag == mid) if tie_up else torch.zeros_like(mag, dtype=torch.bool))
        code += step.to(torch.uint8)
    return code | (torch.signbit(scaled).to(torch.uint8) << 3)


def quantize_nvfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """[rows, cols] float32 -> (packed uint8 [rows, cols/2], scales uint8
    [rows, cols/16], divisor)."""
    w = w.to(torch.float32)
    rows, cols = w.shape
    amax = w.abs().max()
    g = torch.where(amax > 0, amax / torch.tensor(6.0 * 448.0, device=w.device), torch.ones_like(amax))
    blocks = w.reshape(rows, cols // 16, 16)
    bamax = blocks.abs().amax(dim=-1)
    target = (bamax / 6.0) / g
    scales = target.clamp(max=448.0).to(torch.float8_e4m3fn)
    s_val = scales.to(torch.float32)
    denom = s_val * g
    safe = torch.where(denom == 0, torch.ones_like(denom), denom)
    scaled = blocks / safe[..., None]
    scaled = torch.where(denom[..., None] == 0, torch.zeros_like(scaled), scaled)
    codes = e2m1_codes(scaled).reshape(rows, cols)
    packed = codes[:, 0::2] | (codes[:, 1::2] << 4)
    divisor = float((1.0 / g).item())
    return packed.contiguous(), scales.view(torch.uint8).contiguous(), divisor


def _generator(device: torch.device, *key: int) -> torch.Generator:
    seed = 0
    for k in key:
        seed = (seed * 1_000_003 + int(k) + 0x9E3779B9) % (2**63 - 1)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return gen


def bf16_bits(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).view(torch.int16)


@dataclass
class SyntheticLayer:
    router_bf16: torch.Tensor        # int16 bits [E, H] (CPU)
    shared_gate_bf16: torch.Tensor   # int16 bits [H] (CPU)
    router_bias: torch.Tensor | None  # float32 [E] (CPU) or None


def synthetic_router(experts: int, hidden: int, seed: int, layer: int = 0, skew: bool = False) -> SyntheticLayer:
    cpu = torch.device("cpu")
    router = torch.randn(experts, hidden, generator=_generator(cpu, seed, layer, 1), dtype=torch.float32) * 0.02
    gate = torch.randn(hidden, generator=_generator(cpu, seed, layer, 2), dtype=torch.float32) * 0.02
    bias = None
    if skew:
        perm = torch.randperm(experts, generator=_generator(cpu, seed, layer, 5))
        rank = (perm + 1).to(torch.float64)
        bias = (2.0 * torch.log(1.0 / rank.pow(1.2))).to(torch.float32)
    return SyntheticLayer(bf16_bits(router), bf16_bits(gate), bias)


def synthetic_expert_projection(expert: int, projection: int, hidden: int, intermediate: int, seed: int,
                                layer: int = 0, device: str | torch.device = "cuda"):
    """Quantised projection (packed, scales, divisor) of one expert; shapes
    [I, H] for gate/up (projection 0/1) and [H, I] for down (2)."""
    device = torch.device(device)
    shape = (intermediate, hidden) if projection < 2 else (hidden, intermediate)
    gen = _generator(device, seed, layer, 3, expert, projection)
    w = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * 0.02
    return quantize_nvfp4(w)


def synthetic_tokens(tokens: int, hidden: int, seed: int, device: str | torch.device = "cuda") -> torch.Tensor:
    device = torch.device(device)
    gen = _generator(device, seed, 4)
    return torch.randn(tokens, hidden, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def build_bank(runtime, experts: int, hidden: int, intermediate: int, seed: int, layer: int = 0,
               skew: bool = False, device: str | torch.device = "cuda"):
    """Create a MoeBank on `runtime` filled with the seeded synthetic layer.
    Returns (bank, SyntheticLayer)."""
    import numpy as np

    meta = synthetic_router(experts, hidden, seed, layer, skew)
    bank = runtime.create_moe_bank(
        np.ascontiguousarray(meta.router_bf16.numpy().view(np.uint16)),
        np.ascontiguousarray(meta.shared_gate_bf16.numpy().view(np.uint16)),
        intermediate,
    )
    if skew and meta.router_bias is not None:
        bank.set_router_bias(meta.router_bias.numpy())
    keep = []
    for e in range(experts + 1):
        for p in range(3):
            packed, scales, divisor = synthetic_expert_projection(e, p, hidden, intermediate, seed, layer, device)
            if packed.is_cuda:
                # The upload runs on the runtime's own stream: wait for torch's.
                torch.cuda.current_stream(packed.device).synchronize()
                bank.upload_projection_tensor(e, p, packed, scales, divisor)
                keep.append((packed, scales))
            else:
                bank.upload_projection(e, p, packed.numpy(), scales.numpy(), divisor)
        if len(keep) > 96:
            runtime.synchronize()
            keep.clear()
    runtime.synchronize()
    return bank, meta
