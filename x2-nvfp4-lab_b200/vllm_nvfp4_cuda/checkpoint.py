"""Safetensors checkpoint loader for the MoE bank: one layer's router, shared
gate, shared expert and routed experts, streamed shard by shard into a bank.

Two NVFP4 conventions, both read by the lab:

* ModelOpt: ``weight`` (packed E2M1 pairs, uint8 [rows, cols/2]),
  ``weight_scale`` (E4M3 per 16 columns, [rows, cols/16]) and
  ``weight_scale_2`` (an FP32 multiplier; the upload takes its inverse as the
  divisor), native_nvfp4/bench_moe_device_bank.py:33-76 and
  bench_moe_experts.py:37-94;
* compressed-tensors: ``weight_packed``, ``weight_scale`` and
  ``weight_global_scale`` (the divisor itself), native_nvfp4/
  bench_resident_mlp.py:50-62 and probe_native_nvfp4.py:133-141.

Tensor names follow the lab's Qwen3.5-MoE layout under
``model.language_model.layers.{layer}.mlp``: ``gate.weight`` (router, BF16
[experts, hidden]), ``shared_expert_gate.weight`` (BF16 [1, hidden]),
``shared_expert.{gate,up,down}_proj`` and ``experts.{e}.{gate,up,down}_proj``
(bench_moe_routed_layer.py:38-50); the layer's pre-MoE norm is
``model.language_model.layers.{layer}.post_attention_layernorm.weight``
(bench_resident_mlp.py:44-48). A checkpoint is a directory with
``model.safetensors.index.json`` (its ``weight_map`` names each tensor's
shard) or a single ``model.safetensors`` file. Reading needs only the CPU.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def layer_prefix(layer: int) -> str:
    return f"model.language_model.layers.{layer}.mlp"


class CheckpointIndex:
    """Which shard holds each tensor of a safetensors checkpoint."""

    def __init__(self, model_dir):
        self.model_dir = Path(model_dir)
        index = self.model_dir / "model.safetensors.index.json"
        if index.exists():
            self.weight_map = dict(json.loads(index.read_text(encoding="utf-8"))["weight_map"])
        else:
            single = self.model_dir / "model.safetensors"
            if not single.exists():
                raise FileNotFoundError(f"{self.model_dir} has neither model.safetensors.index.json "
                                        "nor model.safetensors")
            from safetensors import safe_open

            with safe_open(single, framework="pt", device="cpu") as f:
                self.weight_map = {k: single.name for k in f.keys()}

    def has(self, key: str) -> bool:
        return key in self.weight_map

    def require(self, keys) -> None:
        missing = [k for k in keys if k not in self.weight_map]
        if missing:
            raise KeyError(f"checkpoint index is missing {missing[0]}")

    def read(self, keys) -> dict:
        """The tensors named by ``keys`` (torch, CPU), opening each shard once."""
        from safetensors import safe_open

        keys = list(keys)
        self.require(keys)
        by_shard: dict[str, list[str]] = {}
        for k in keys:
            by_shard.setdefault(self.weight_map[k], []).append(k)
        out = {}
        for shard, shard_keys in by_shard.items():
            with safe_open(self.model_dir / shard, framework="pt", device="cpu") as f:
                for k in shard_keys:
                    out[k] = f.get_tensor(k)
        return out


@dataclass(frozen=True)
class ProjectionKeys:
    convention: str  # "modelopt" or "compressed-tensors"
    packed: str
    scales: str
    scale: str

    def keys(self) -> tuple[str, str, str]:
        return (self.packed, self.scales, self.scale)


def projection_keys(index: CheckpointIndex, base: str) -> ProjectionKeys:
    """The tensor names of one NVFP4 projection (``base`` = ``...{proj}``)."""
    if index.has(base + ".weight_packed"):
        return ProjectionKeys("compressed-tensors", base + ".weight_packed", base + ".weight_scale",
                              base + ".weight_global_scale")
    if index.has(base + ".weight"):
        return ProjectionKeys("modelopt", base + ".weight", base + ".weight_scale", base + ".weight_scale_2")
    raise KeyError(f"checkpoint index has no NVFP4 weight for {base}")


def _u8(t) -> np.ndarray:
    import torch

    if t.dtype == torch.uint8:
        return np.ascontiguousarray(t.numpy())
    if t.element_size() == 1:  # float8_e4m3fn scales, int8 packs: the same bytes
        return np.ascontiguousarray(t.view(torch.uint8).numpy())
    raise ValueError(f"expected one-byte elements, got {t.dtype}")


def _bf16_bits(t) -> np.ndarray:
    import torch

    if t.dtype != torch.bfloat16:
        raise ValueError(f"expected bfloat16, got {t.dtype}")
    return np.ascontiguousarray(t.contiguous().view(torch.int16).numpy().view(np.uint16))


def projection_arrays(keys: ProjectionKeys, tensors: dict) -> tuple[np.ndarray, np.ndarray, float]:
    """(packed, scales, divisor) of one projection, as ``MoeBank.upload_projection`` takes them."""
    packed = _u8(tensors[keys.packed])
    scales = _u8(tensors[keys.scales])
    value = float(tensors[keys.scale].float().reshape(-1)[0])
    if not math.isfinite(value) or value <= 0.0:
        raise ValueError(f"invalid {keys.scale}: {value}")
    divisor = 1.0 / value if keys.convention == "modelopt" else value
    return packed, scales, divisor


@dataclass
class LayerCheckpoint:
    """A layer's routing weights and NVFP4 projections: ``projections[e]`` =
    [(packed, scales, divisor)] * 3 for gate, up, down; index ``experts`` is
    the shared expert."""

    experts: int
    hidden: int
    intermediate: int
    router_bf16: np.ndarray
    shared_gate_bf16: np.ndarray
    conventions: set = field(default_factory=set)
    projections: dict = field(default_factory=dict)


def _expert_base(layer: int, expert: int, experts: int) -> str:
    p = layer_prefix(layer)
    return p + ".shared_expert" if expert == experts else p + f".experts.{expert}"


def read_routing(index: CheckpointIndex, layer: int) -> tuple[np.ndarray, np.ndarray]:
    """Router BF16 bits [experts, hidden] and shared gate BF16 bits [hidden]."""
    p = layer_prefix(layer)
    t = index.read([p + ".gate.weight", p + ".shared_expert_gate.weight"])
    router = _bf16_bits(t[p + ".gate.weight"])
    shared_gate = _bf16_bits(t[p + ".shared_expert_gate.weight"]).reshape(-1)
    if router.ndim != 2 or shared_gate.size != router.shape[1]:
        raise ValueError(f"router {router.shape} and shared gate {shared_gate.shape} disagree")
    return router, np.ascontiguousarray(shared_gate)


def stream_layer(index: CheckpointIndex, layer: int, experts: int, sink, expert_ids=None) -> set:
    """Call ``sink(expert, projection, packed, scales, divisor)`` for every
    projection of the listed experts (default: every routed expert and the
    shared one), grouped by shard so each shard is opened once and only one
    shard's tensors are held at a time. Returns the conventions seen."""
    from safetensors import safe_open

    ids = list(range(experts + 1)) if expert_ids is None else list(expert_ids)
    plan = {}
    for e in ids:
        for pi, proj in enumerate(PROJECTIONS):
            k = projection_keys(index, _expert_base(layer, e, experts) + "." + proj)
            index.require(k.keys())
            plan[(e, pi)] = k
    # Grouped by the shard of each projection's packed tensor; a scale kept in
    # another shard is fetched through the index.
    by_shard: dict[str, list[tuple[int, int]]] = {}
    for ep, k in plan.items():
        by_shard.setdefault(index.weight_map[k.packed], []).append(ep)
    conventions = set()
    for shard, eps in by_shard.items():
        names = {name for ep in eps for name in plan[ep].keys()}
        local = [n for n in names if index.weight_map[n] == shard]
        with safe_open(index.model_dir / shard, framework="pt", device="cpu") as f:
            tensors = {n: f.get_tensor(n) for n in local}
        remote = names.difference(local)
        if remote:
            tensors.update(index.read(remote))
        for e, pi in eps:
            k = plan[(e, pi)]
            conventions.add(k.convention)
            sink(e, pi, *projection_arrays(k, tensors))
    return conventions


def read_layer(model_dir, layer: int, expert_ids=None) -> LayerCheckpoint:
    """The whole layer in host memory (tests and small models; ``load_bank``
    streams instead)."""
    index = CheckpointIndex(model_dir)
    router, shared_gate = read_routing(index, layer)
    experts, hidden = router.shape
    out = LayerCheckpoint(experts, hidden, 0, router, shared_gate)

    def sink(e, p, packed, scales, divisor):
        out.projections.setdefault(e, [None, None, None])[p] = (packed, scales, divisor)

    out.conventions = stream_layer(index, layer, experts, sink, expert_ids)
    shared = out.projections.get(experts)
    any_expert = shared if shared is not None else next(iter(out.projections.values()))
    out.intermediate = int(any_expert[0][0].shape[0])
    return out


def read_norm_weight(model_dir, layer: int) -> np.ndarray | None:
    """BF16 bits [hidden] of the layer's pre-MoE RMSNorm weight, or None if absent."""
    index = CheckpointIndex(model_dir)
    key = f"model.language_model.layers.{layer}.post_attention_layernorm.weight"
    if not index.has(key):
        return None
    t = index.read([key])[key]
    import torch

    if t.dtype != torch.bfloat16:
        t = t.float().to(torch.bfloat16)
    return _bf16_bits(t).reshape(-1)


def load_bank(runtime, model_dir, layer: int):
    """Create a bank on ``runtime`` from checkpoint layer ``layer`` and stream
    every expert into it (``MoeBank.upload_projection`` per projection, shard
    by shard). Returns (bank, info) with info = {"experts", "hidden",
    "intermediate", "conventions", "payload_bytes"}."""
    index = CheckpointIndex(model_dir)
    router, shared_gate = read_routing(index, layer)
    experts, hidden = router.shape
    shared_gate_keys = projection_keys(index, _expert_base(layer, experts, experts) + ".gate_proj")
    index.require(shared_gate_keys.keys())
    intermediate = int(index.read([shared_gate_keys.packed])[shared_gate_keys.packed].shape[0])
    bank = runtime.create_moe_bank(router, shared_gate, intermediate)
    payload = [0]

    def sink(e, p, packed, scales, divisor):
        bank.upload_projection(e, p, packed, scales, divisor)
        payload[0] += packed.nbytes + scales.nbytes

    try:
        conventions = stream_layer(index, layer, experts, sink)
    except Exception:
        bank.close()
        raise
    return bank, {"experts": experts, "hidden": hidden, "intermediate": intermediate,
                  "conventions": sorted(conventions), "payload_bytes": payload[0]}


def load_stack(runtime, model_dir, layers, epsilon: float = 1e-6, device: str = "cuda"):
    """A resident layer stack (vllm_nvfp4_cuda.stack.MoeStack) of checkpoint
    layers: each layer's bank (``load_bank``) and its pre-MoE RMSNorm weight
    (``post_attention_layernorm.weight``; ones where the checkpoint has
    none), fused into each layer's forward."""
    import torch

    from .stack import MoeStack

    banks, norms = [], []
    try:
        for layer in layers:
            bank, info = load_bank(runtime, model_dir, layer)
            banks.append(bank)
            bits = read_norm_weight(model_dir, layer)
            if bits is None:
                bits = np.full(info["hidden"], 0x3F80, dtype=np.uint16)  # BF16 1.0
            norms.append(torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device))
        return MoeStack(runtime, banks, epsilon=epsilon, norm_weights=norms)
    except Exception:
        for bank in banks:
            bank.close()
        raise
