"""Expert parallelism of the NVFP4 MoE layer: one process per GPU.

Rank r of N computes the routed experts [r*E/N, (r+1)*E/N) and, on rank 0,
the shared expert. The router is replicated and every rank routes every token
(the routing kernels are deterministic, so every rank gets the same ids,
weights and permutation); the tokens are replicated too. Each rank writes the
FP32 partial sum of its experts (plus the residual on rank 0), a sum
all-reduce over the ranks (NCCL over NVLink on GPUs) adds the partials, and
``finalize_bf16`` rounds the sum to BF16. This is the batch-1 decode scheme
of an expert-parallel layer (one exchange of [tokens, hidden] FP32 per
layer); it serves prefill the same way, with every rank routing all tokens.

The lab itself runs on one device and has no counterpart of this module.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ExpertRange:
    first: int
    count: int
    shared_here: bool


def expert_range(rank: int, world: int, experts: int) -> ExpertRange:
    """Routed experts owned by ``rank`` of ``world``; the shared expert is on rank 0."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if experts % world != 0:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return ExpertRange(rank * per, per, rank == 0)


class ExpertParallelLayer:
    """A bank that computes one rank's expert range, plus the reduction.

    ``bank`` needs ``experts``, ``set_expert_range`` and ``forward_partial``
    (vllm_nvfp4_cuda.runtime.MoeBank); ``finalize`` turns the reduced FP32
    sum into the BF16 output (Runtime.finalize_bf16 on GPUs). ``group`` is a
    torch.distributed process group (None: the default group).

    With ``fused_runtime`` (a Runtime; GPUs only) calls of up to 64 tokens use
    the combine fused with the reduction over NVLink peer memory
    (MoeBank.forward_ep); every rank's buffers are mapped by every other rank
    through CUDA IPC handles exchanged here. Larger calls use the collective.
    """

    def __init__(self, bank, finalize, group=None, fused_runtime=None):
        import torch.distributed as dist

        self.bank = bank
        self.finalize = finalize
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.range = expert_range(self.rank, self.world, bank.experts)
        bank.set_expert_range(self.range.first, self.range.count, self.range.shared_here)
        self.ep = None
        if fused_runtime is not None:
            from vllm_nvfp4_cuda.runtime import EpContext

            self.ep = EpContext(fused_runtime, self.rank, self.world, 64, bank.hidden)
            handles = [None] * self.world
            dist.all_gather_object(handles, self.ep.ipc_handle(), group=group)
            self.ep.open_peers(handles)
            dist.barrier(group=group)

    def close(self):
        if self.ep is not None:
            self.ep.close()
            self.ep = None

    def partial(self, x, residual=None, stream=None):
        """This rank's FP32 partial sum (the residual is added on rank 0 only)."""
        return self.bank.forward_partial(x, residual=residual if self.rank == 0 else None, stream=stream)

    def forward(self, x, residual=None, stream=None):
        """Layer output (BF16 on GPUs) on every rank. On GPUs the partial,
        the all-reduce and the finalize are all ordered on ``stream`` (a
        torch.cuda.Stream; None: torch's current stream)."""
        import contextlib

        import torch
        import torch.distributed as dist

        if self.ep is not None and x.shape[0] <= self.ep.max_tokens:
            return self.bank.forward_ep(self.ep, x, residual=residual, stream=stream)
        ctx = torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()
        with ctx:
            part = self.partial(x, residual)
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            return self.finalize(part)
