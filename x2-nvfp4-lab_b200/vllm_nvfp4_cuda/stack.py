"""Resident multi-layer MoE decode stack (attention omitted).

Each layer l maps the hidden state h (BF16 [tokens, hidden]) to

    h <- BF16(h + MoE_l(RMSNorm_l(h)))

with the pre-norm a BF16 RMSNorm (FP32 statistic, epsilon 1e-6, weight ones
unless given) and the MoE layer one bank's forward with h as its residual.
This is the lab's full-model decode step (native_nvfp4/bench_moe_full_model.py:
366-406: per layer ``rmsnorm_device``, ``bank.decode_device``, ``add_device``)
without its attention blocks, at the hidden-state precision of the BF16
forward path. All layers stay resident in HBM. By default each layer is one
bank forward with the RMSNorm fused in (NVFP4_MOE_PRE_NORM: the routing
kernel normalises its staged copy of the tokens, with the same bits as the
standalone RMSNorm); ``fused_norm=False`` runs the standalone RMSNorm before
each layer instead. ``capture`` records a step once in a CUDA graph so a step
is a single graph launch.
"""

from __future__ import annotations


class MoeStack:
    """``banks``: MoeBank objects of one runtime, one per layer, same hidden size.
    ``norm_weights``: optional BF16 CUDA tensors [hidden] per layer (ones when None).
    With ``fused_norm`` each bank is given its layer's norm (``set_pre_norm``)."""

    def __init__(self, runtime, banks, epsilon: float = 1e-6, norm_weights=None, fused_norm: bool = True):
        import torch

        self.runtime = runtime
        self.banks = list(banks)
        if not self.banks:
            raise ValueError("a stack needs at least one bank")
        self.hidden = self.banks[0].hidden
        if any(b.hidden != self.hidden for b in self.banks):
            raise ValueError("every bank of a stack must have the same hidden size")
        self.epsilon = float(epsilon)
        if norm_weights is None:
            ones = torch.ones(self.hidden, dtype=torch.bfloat16, device="cuda")
            norm_weights = [ones] * len(self.banks)
        if len(norm_weights) != len(self.banks):
            raise ValueError("one norm weight per layer")
        self.norm_weights = [w.contiguous() for w in norm_weights]
        self.fused_norm = bool(fused_norm)
        if self.fused_norm:
            for bank, w in zip(self.banks, self.norm_weights):
                bank.set_pre_norm(w, self.epsilon)

    @property
    def layers(self) -> int:
        return len(self.banks)

    def _enqueue(self, h, scratch, normed, stream):
        """Run every layer from h; returns the tensor holding the final state
        (h or scratch: the two alternate as layer input and output)."""
        a, b = h, scratch
        for bank, w in zip(self.banks, self.norm_weights):
            if self.fused_norm:
                bank.forward(a, residual=a, out=b, stream=stream, pre_norm=True)
            else:
                self.runtime.rmsnorm_bf16(a, w, self.epsilon, out=normed, stream=stream)
                bank.forward(normed, residual=a, out=b, stream=stream)
            a, b = b, a
        return a

    def forward(self, x, stream=None):
        """The stack applied to x (CUDA bfloat16 [tokens, hidden]); returns a new tensor."""
        import torch

        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("x must be a CUDA bfloat16 tensor [tokens, hidden]")
        h = x.contiguous().clone()
        scratch = torch.empty_like(h)
        normed = torch.empty_like(h)
        return self._enqueue(h, scratch, normed, stream)

    def capture(self, tokens: int, warmup: int = 2):
        """A CUDA graph of one step over ``tokens`` tokens (see StackGraph)."""
        return StackGraph(self, tokens, warmup)


class StackGraph:
    """One captured step: write the step's tokens into ``input`` (or pass them to
    ``run``), ``replay()``, read ``output``. The graph owns its buffers, so the
    input survives the step and ``output`` is overwritten by the next replay."""

    def __init__(self, stack: MoeStack, tokens: int, warmup: int = 2):
        import torch

        if tokens < 1:
            raise ValueError("tokens must be positive")
        self.stack = stack
        H = stack.hidden
        self.input = torch.zeros(tokens, H, dtype=torch.bfloat16, device="cuda")
        self._h = torch.empty_like(self.input)
        self._scratch = torch.empty_like(self.input)
        self._normed = torch.empty_like(self.input)
        self.stream = torch.cuda.Stream()
        self.stream.wait_stream(torch.cuda.current_stream())
        # Eager passes first: every kernel's one-time launch setup (shared-memory
        # limits, occupancy queries) happens outside the capture.
        with torch.cuda.stream(self.stream):
            for _ in range(max(1, warmup)):
                self._h.copy_(self.input)
                self.stack._enqueue(self._h, self._scratch, self._normed, self.stream)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._h.copy_(self.input)
            self.output = self.stack._enqueue(self._h, self._scratch, self._normed, self.stream)
        torch.cuda.current_stream().wait_stream(self.stream)

    def replay(self):
        self.graph.replay()
        return self.output

    def run(self, x):
        """Copy x into the input buffer and replay; returns ``output``."""
        self.input.copy_(x)
        return self.replay()

    def close(self):
        self.graph = None
