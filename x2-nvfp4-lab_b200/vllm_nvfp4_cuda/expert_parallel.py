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
``TokenShardedLayer`` is the other form: each rank brings its own tokens and
all-to-alls move token rows to the ranks owning their experts and the FP32
partials back.

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


class TokenShardedLayer:
    """Expert parallelism with the tokens sharded over the ranks (prefill and
    batched decode), as a host-level composition of the bank forward and
    ``torch.distributed`` all-to-alls.

    Each rank brings its own tokens. The router and the shared expert are
    replicated; rank r owns the routed experts ``expert_range(r, N, E)``.
    Per call:

    1. the rank's partial sum of its own tokens: its routed experts, the
       shared expert and the residual (``forward_partial``), which also routes
       them (``last_routing``);
    2. a counts all-to-all, then a payload all-to-all of the token rows, each
       token sent once to every other rank that owns one of its eight picks;
    3. each rank's partial sums of the tokens it received (its routed experts
       only; it routes them again, to the same picks);
    4. the partials all-to-all back, then the sum at the origin in rank
       order, and ``finalize``.

    ``bank`` needs ``experts``, ``set_expert_range``, ``forward_partial`` and
    ``last_routing`` (vllm_nvfp4_cuda.runtime.MoeBank, with the shared
    expert and the rank's routed experts uploaded); ``finalize`` turns the
    FP32 sum into the output (Runtime.finalize_bf16 on GPUs). Calls route
    at most 16384 tokens per rank (the bank keeps the routing record of
    calls that run as one pass). The device kernels are those of the bank;
    this class only moves rows between ranks (NCCL on GPUs)."""

    def __init__(self, bank, finalize, group=None):
        import torch.distributed as dist

        self.bank = bank
        self.finalize = finalize
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.range = expert_range(self.rank, self.world, bank.experts)
        self.per_rank = bank.experts // self.world

    def _exchange(self, send, send_counts, recv_counts):
        import torch
        import torch.distributed as dist

        out = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
        dist.all_to_all_single(out, send.contiguous(), output_split_sizes=list(recv_counts),
                               input_split_sizes=list(send_counts), group=self.group)
        return out

    def forward(self, x, residual=None):
        """Layer output of this rank's tokens ``x`` [tokens, hidden] (BF16 on
        GPUs), with ``residual`` added; every rank must call it, with its own
        token count (zero allowed)."""
        import numpy as np
        import torch
        import torch.distributed as dist

        T = x.shape[0]
        first, count = self.range.first, self.range.count
        # 1. Own tokens: own routed experts + shared expert + residual.
        self.bank.set_expert_range(first, count, True)
        if T > 0:
            part = self.bank.forward_partial(x, residual=residual)
            if x.is_cuda:
                torch.cuda.current_stream(x.device).synchronize()
            ids = np.asarray(self.bank.last_routing(T).ids)[:, :8]
        else:
            part = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
            ids = np.zeros((0, 8), dtype=np.int64)
        # 2. Destinations: every other rank owning one of a token's picks.
        owner = ids // self.per_rank
        idx = [np.nonzero((owner == k).any(axis=1))[0] if k != self.rank else np.zeros(0, dtype=np.int64)
               for k in range(self.world)]
        send_counts = [len(i) for i in idx]
        counts = torch.tensor(send_counts, dtype=torch.int64, device=x.device)
        recv = torch.empty_like(counts)
        dist.all_to_all_single(recv, counts, group=self.group)
        recv_counts = recv.tolist()
        order = torch.from_numpy(np.concatenate(idx).astype(np.int64)).to(x.device)
        recv_x = self._exchange(x.index_select(0, order), send_counts, recv_counts)
        # 3. Received tokens: own routed experts only.
        self.bank.set_expert_range(first, count, False)
        if recv_x.shape[0] > 0:
            recv_part = self.bank.forward_partial(recv_x)
        else:
            recv_part = torch.zeros(recv_x.shape, dtype=torch.float32, device=x.device)
        self.bank.set_expert_range(first, count, True)
        # 4. Partials back; the sum in rank order at the origin.
        back = self._exchange(recv_part, recv_counts, send_counts)
        out = torch.zeros(part.shape, dtype=torch.float32, device=x.device)
        start = 0
        for k in range(self.world):
            if k == self.rank:
                out += part
            elif send_counts[k]:
                sel = torch.from_numpy(idx[k].astype(np.int64)).to(x.device)
                out.index_add_(0, sel, back[start:start + send_counts[k]])
            start += send_counts[k]
        return self.finalize(out)
