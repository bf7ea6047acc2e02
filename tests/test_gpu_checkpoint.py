"""A bank loaded from a safetensors checkpoint (vllm_nvfp4_cuda.checkpoint)
computes the oracle's layer (needs an sm_100a GPU)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor

pytestmark = pytest.mark.gpu


def test_checkpoint_bank_matches_oracle(cuda_runtime, tmp_path):
    import torch
    from safetensors.torch import save_file

    from vllm_nvfp4_cuda.checkpoint import load_bank

    E, H, I = 8, 256, 128
    host = synthetic_np.make_bank(E, H, I, 31)

    def bf16(bits):
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)

    p = "model.language_model.layers.0.mlp"
    t = {p + ".gate.weight": bf16(host.router_bf16), p + ".shared_expert_gate.weight": bf16(
        host.shared_gate_bf16.reshape(1, -1))}
    for e in range(E + 1):
        base = p + (".shared_expert" if e == E else f".experts.{e}")
        for pi, name in enumerate(("gate_proj", "up_proj", "down_proj")):
            m = host.projections[pi][e]
            t[f"{base}.{name}.weight_packed"] = torch.from_numpy(m.packed.copy())
            t[f"{base}.{name}.weight_scale"] = torch.from_numpy(m.scales.copy()).view(torch.float8_e4m3fn)
            t[f"{base}.{name}.weight_global_scale"] = torch.tensor([m.global_scale], dtype=torch.float32)
    save_file(t, str(tmp_path / "model.safetensors"))

    bank, info = load_bank(cuda_runtime, tmp_path, 0)
    try:
        assert (info["experts"], info["hidden"], info["intermediate"]) == (E, H, I)
        xbits = synthetic_np.tokens_bf16(3, H, 5)
        rbits = synthetic_np.tokens_bf16(3, H, 6)
        out = bank.forward(bits_to_bf16_tensor(xbits), residual=bits_to_bf16_tensor(rbits))
        torch.cuda.synchronize()
        got = bf16_tensor_to_f32(out)
        ref = moe_layer(host, synthetic_np.bf16_bits_to_f32(xbits), synthetic_np.bf16_bits_to_f32(rbits))
        assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
        assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    finally:
        bank.close()
