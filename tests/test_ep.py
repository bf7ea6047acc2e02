"""Expert-parallel host logic on CPU: the expert partition and a two-rank
``gloo`` run of ExpertParallelLayer whose banks are the oracle's partial
layer (the device kernels are covered by tests/test_gpu_ep.py).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from vllm_nvfp4_cuda.expert_parallel import ExpertParallelLayer, TokenShardedLayer, expert_range


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_range_covers_every_expert_once(world):
    E = 256
    seen = np.zeros(E, dtype=int)
    shared = 0
    for r in range(world):
        rng = expert_range(r, world, E)
        seen[rng.first:rng.first + rng.count] += 1
        shared += int(rng.shared_here)
    assert (seen == 1).all()
    assert shared == 1 and expert_range(0, world, E).shared_here


def test_expert_range_rejects_uneven_and_bad_rank():
    with pytest.raises(ValueError):
        expert_range(0, 3, 256)
    with pytest.raises(ValueError):
        expert_range(2, 2, 256)


class _OracleBank:
    """Stands in for MoeBank: forward_partial is the oracle's partial layer."""

    def __init__(self, host):
        self.host = host
        self.experts = host.experts
        self.range = None

    def set_expert_range(self, first, count, shared_here):
        self.range = (first, count, shared_here)

    def forward_partial(self, x, residual=None, stream=None):
        import torch

        from oracle.nvfp4_oracle import moe_layer

        first, count, shared_here = self.range
        r = residual.numpy() if residual is not None else None
        result = moe_layer(self.host, x.numpy(), r, expert_range=(first, count), shared_here=shared_here)
        self.last_ids = result.ids
        return torch.from_numpy(result.out.astype(np.float32))

    def last_routing(self, tokens):
        from types import SimpleNamespace

        return SimpleNamespace(ids=self.last_ids[:tokens])


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    from oracle import synthetic_np

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        host = synthetic_np.make_bank(16, 256, 128, 41)
        x = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(5, 256, 42))
        res = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(5, 256, 43))
        layer = ExpertParallelLayer(_OracleBank(host), finalize=lambda t: t)
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(res))
        if rank == 0:
            np.save(result_path, out.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_layer_matches_single_device(tmp_path):
    import torch.multiprocessing as mp

    from oracle import synthetic_np
    from oracle.nvfp4_oracle import moe_layer

    result = tmp_path / "ep_out.npy"
    mp.start_processes(_worker, args=(2, _free_port(), str(result)), nprocs=2, start_method="spawn", join=True)
    got = np.load(result)
    host = synthetic_np.make_bank(16, 256, 128, 41)
    x = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(5, 256, 42))
    res = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(5, 256, 43))
    ref = moe_layer(host, x, res).out
    # Only the order of the FP32 additions differs.
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


def _rank_tokens(rank):
    from oracle import synthetic_np

    T = 0 if rank == 2 else 3 + 2 * rank
    x = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(T, 256, 60 + rank))
    res = synthetic_np.bf16_bits_to_f32(synthetic_np.tokens_bf16(T, 256, 80 + rank))
    return x, res


def _sharded_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    from oracle import synthetic_np

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        host = synthetic_np.make_bank(16, 256, 128, 41)
        x, res = _rank_tokens(rank)
        layer = TokenShardedLayer(_OracleBank(host), finalize=lambda t: t)
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(res))
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_token_sharded_layer_matches_single_device(tmp_path, world):
    """Tokens sharded over the ranks (uneven counts, one rank without tokens
    at four ranks), experts split, rows and partials moved by all-to-alls:
    every rank gets the single-device layer output of its own tokens."""
    import torch.multiprocessing as mp

    from oracle import synthetic_np
    from oracle.nvfp4_oracle import moe_layer

    mp.start_processes(_sharded_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    host = synthetic_np.make_bank(16, 256, 128, 41)
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npy")
        x, res = _rank_tokens(rank)
        assert got.shape == x.shape
        if x.shape[0] == 0:
            continue
        ref = moe_layer(host, x, res).out
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
