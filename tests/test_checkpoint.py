"""Safetensors checkpoint loader (vllm_nvfp4_cuda.checkpoint), on CPU.

Synthetic checkpoints are written from the oracle's quantised banks in both
NVFP4 conventions the lab reads (ModelOpt: weight / weight_scale /
weight_scale_2; compressed-tensors: weight_packed / weight_scale /
weight_global_scale), sharded with an index or as a single file, and read
back: router and shared-gate bits, packed codes and scale bytes must be the
written ones, and the divisor the one the lab passes to its upload (the
inverse of weight_scale_2, or weight_global_scale itself).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import synthetic_np

E, H, I = 8, 128, 64
PROJ = ("gate_proj", "up_proj", "down_proj")


def _bf16(bits: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _tensors(bank, layer: int, convention: str) -> dict:
    import torch

    p = f"model.language_model.layers.{layer}.mlp"
    out = {p + ".gate.weight": _bf16(bank.router_bf16), p + ".shared_expert_gate.weight": _bf16(
        bank.shared_gate_bf16.reshape(1, -1))}
    out[f"model.language_model.layers.{layer}.post_attention_layernorm.weight"] = _bf16(
        synthetic_np.bf16_bits_from_f32(np.linspace(0.5, 1.5, H, dtype=np.float32)))
    for e in range(E + 1):
        base = p + (".shared_expert" if e == E else f".experts.{e}")
        for pi, name in enumerate(PROJ):
            m = bank.projections[pi][e]
            scales = torch.from_numpy(m.scales.copy()).view(torch.float8_e4m3fn)
            if convention == "modelopt":
                out[f"{base}.{name}.weight"] = torch.from_numpy(m.packed.copy())
                out[f"{base}.{name}.weight_scale"] = scales
                out[f"{base}.{name}.weight_scale_2"] = torch.tensor(1.0 / m.global_scale, dtype=torch.float32)
            else:
                out[f"{base}.{name}.weight_packed"] = torch.from_numpy(m.packed.copy())
                out[f"{base}.{name}.weight_scale"] = scales
                out[f"{base}.{name}.weight_global_scale"] = torch.tensor([m.global_scale], dtype=torch.float32)
    return out


def _write_sharded(tmp_path, tensors: dict, layer: int) -> None:
    from safetensors.torch import save_file

    p = f"model.language_model.layers.{layer}.mlp"
    shard_of = {}
    for k in tensors:
        second = any(f".experts.{e}." in k for e in range(4, E)) or ".shared_expert." in k
        shard_of[k] = "model-00002-of-00002.safetensors" if second else "model-00001-of-00002.safetensors"
    # One projection keeps its scale in the other shard.
    shard_of[p + ".experts.1.down_proj.weight_scale"] = "model-00002-of-00002.safetensors"
    for shard in set(shard_of.values()):
        save_file({k: v for k, v in tensors.items() if shard_of[k] == shard}, str(tmp_path / shard))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": shard_of}))


@pytest.fixture(scope="module")
def bank_host():
    return synthetic_np.make_bank(E, H, I, 23)


def _check_layer(layer_ckpt, bank, convention: str) -> None:
    np.testing.assert_array_equal(layer_ckpt.router_bf16, bank.router_bf16)
    np.testing.assert_array_equal(layer_ckpt.shared_gate_bf16, bank.shared_gate_bf16)
    assert (layer_ckpt.experts, layer_ckpt.hidden, layer_ckpt.intermediate) == (E, H, I)
    assert layer_ckpt.conventions == {convention}
    for e in range(E + 1):
        for pi in range(3):
            m = bank.projections[pi][e]
            packed, scales, divisor = layer_ckpt.projections[e][pi]
            np.testing.assert_array_equal(packed, m.packed)
            np.testing.assert_array_equal(scales, m.scales)
            stored = float(np.float32(1.0 / m.global_scale if convention == "modelopt" else m.global_scale))
            assert divisor == (1.0 / stored if convention == "modelopt" else stored)


def test_read_layer_modelopt_sharded(tmp_path, bank_host):
    from vllm_nvfp4_cuda.checkpoint import read_layer

    _write_sharded(tmp_path, _tensors(bank_host, 3, "modelopt"), 3)
    _check_layer(read_layer(tmp_path, 3), bank_host, "modelopt")


def test_read_layer_compressed_tensors_single_file(tmp_path, bank_host):
    from safetensors.torch import save_file

    from vllm_nvfp4_cuda.checkpoint import read_layer, read_norm_weight

    save_file(_tensors(bank_host, 0, "compressed-tensors"), str(tmp_path / "model.safetensors"))
    _check_layer(read_layer(tmp_path, 0), bank_host, "compressed-tensors")
    w = read_norm_weight(tmp_path, 0)
    np.testing.assert_array_equal(w, synthetic_np.bf16_bits_from_f32(np.linspace(0.5, 1.5, H, dtype=np.float32)))
    assert read_norm_weight(tmp_path, 1) is None


class _RecordingBank:
    def __init__(self, hidden=H):
        self.uploads = {}
        self.closed = False
        self.hidden = hidden
        self.pre_norm = None

    def set_pre_norm(self, weight, epsilon):
        self.pre_norm = (weight, epsilon)

    def upload_projection(self, e, p, packed, scales, divisor):
        assert (e, p) not in self.uploads
        self.uploads[(e, p)] = (packed, scales, divisor)

    def close(self):
        self.closed = True


class _RecordingRuntime:
    def __init__(self):
        self.created = None
        self.bank = _RecordingBank()
        self.banks = []

    def create_moe_bank(self, router, shared_gate, intermediate):
        self.created = (router, shared_gate, intermediate)
        self.bank = _RecordingBank()
        self.banks.append(self.bank)
        return self.bank


def test_load_bank_streams_every_projection(tmp_path, bank_host):
    from vllm_nvfp4_cuda.checkpoint import load_bank

    _write_sharded(tmp_path, _tensors(bank_host, 2, "modelopt"), 2)
    rt = _RecordingRuntime()
    bank, info = load_bank(rt, tmp_path, 2)
    assert bank is rt.bank and not bank.closed
    router, shared_gate, intermediate = rt.created
    np.testing.assert_array_equal(router, bank_host.router_bf16)
    np.testing.assert_array_equal(shared_gate, bank_host.shared_gate_bf16)
    assert intermediate == I
    assert set(bank.uploads) == {(e, p) for e in range(E + 1) for p in range(3)}
    for (e, p), (packed, scales, _) in bank.uploads.items():
        np.testing.assert_array_equal(packed, bank_host.projections[p][e].packed)
        np.testing.assert_array_equal(scales, bank_host.projections[p][e].scales)
    assert info["experts"] == E and info["hidden"] == H and info["intermediate"] == I
    assert info["conventions"] == ["modelopt"]
    assert info["payload_bytes"] == (E + 1) * 3 * (H * I // 2 + H * I // 16)


def test_missing_tensor_and_bad_scale(tmp_path, bank_host):
    from safetensors.torch import save_file

    import torch

    from vllm_nvfp4_cuda.checkpoint import load_bank, read_layer

    t = _tensors(bank_host, 0, "modelopt")
    key = "model.language_model.layers.0.mlp.experts.5.up_proj.weight_scale"
    del t[key]
    save_file(t, str(tmp_path / "model.safetensors"))
    with pytest.raises(KeyError, match="experts.5.up_proj.weight_scale"):
        read_layer(tmp_path, 0)

    t = _tensors(bank_host, 0, "modelopt")
    t["model.language_model.layers.0.mlp.experts.2.gate_proj.weight_scale_2"] = torch.tensor(0.0)
    (tmp_path / "model.safetensors").unlink()
    save_file(t, str(tmp_path / "model.safetensors"))
    rt = _RecordingRuntime()
    with pytest.raises(ValueError, match="weight_scale_2"):
        load_bank(rt, tmp_path, 0)
    assert rt.bank.closed


def test_missing_checkpoint(tmp_path):
    from vllm_nvfp4_cuda.checkpoint import CheckpointIndex

    with pytest.raises(FileNotFoundError):
        CheckpointIndex(tmp_path)


def test_load_stack_uses_each_layers_norm(tmp_path, bank_host):
    """load_stack: one bank per layer plus its post-attention norm weight
    (ones for a layer without one), handed to each bank as its fused pre-norm."""
    import torch
    from safetensors.torch import save_file

    from vllm_nvfp4_cuda.checkpoint import load_stack

    t = _tensors(bank_host, 0, "compressed-tensors")
    t1 = _tensors(bank_host, 1, "compressed-tensors")
    del t1["model.language_model.layers.1.post_attention_layernorm.weight"]
    t.update({k: v.clone() for k, v in t1.items()})  # safetensors refuses shared storage
    save_file(t, str(tmp_path / "model.safetensors"))
    rt = _RecordingRuntime()
    stack = load_stack(rt, tmp_path, [0, 1], epsilon=1e-5, device="cpu")
    assert stack.layers == 2 and stack.fused_norm and stack.banks == rt.banks
    w0, eps0 = rt.banks[0].pre_norm
    w1, eps1 = rt.banks[1].pre_norm
    assert eps0 == eps1 == 1e-5
    np.testing.assert_array_equal(w0.view(torch.int16).numpy().view(np.uint16),
                                  synthetic_np.bf16_bits_from_f32(np.linspace(0.5, 1.5, H, dtype=np.float32)))
    assert (w1.float() == 1.0).all()
    assert all(len(b.uploads) == (E + 1) * 3 for b in rt.banks)
