"""BASELINE config 4 at its shape: a resident stack of four full-size layers
(256 x 512 experts, hidden 2048, GPU-generated seeded banks), each
h <- BF16(h + MoE(RMSNorm(h))) with the RMSNorm fused into the layer call,
at batch 1 and batch 64 (needs an sm_100a GPU).

* Per-layer synchronised calls give every layer's input and output; the
  captured graph of the whole step must reproduce the last layer's output
  bit for bit (the lab's composition oracle: queued multi-layer output equals
  the per-layer synchronised replay, BENCHMARKS.md:607-609).
* Each layer is checked against the oracle on that layer's GPU input: the
  RMSNorm bits are those of the standalone RMSNorm kernel (the fused norm is
  tested bit-identical to it elsewhere), routing ids of every token equal the
  C restatement's, and the layer output meets the BASELINE bound against the
  FP32 dequantise-then-matmul oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cpu_oracle
from oracle.nvfp4_oracle import BankHost, QuantizedMatrix, max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL

pytestmark = pytest.mark.gpu

E, H, I = 256, 2048, 512
LAYERS = 4
SEED = 0


@pytest.fixture(scope="module")
def full_stack(cuda_runtime):
    from vllm_nvfp4_cuda import synthetic
    from vllm_nvfp4_cuda.stack import MoeStack

    built = [synthetic.build_bank(cuda_runtime, E, H, I, SEED, layer=101 + layer) for layer in range(LAYERS)]
    banks = [b for b, _ in built]
    metas = [m for _, m in built]
    yield MoeStack(cuda_runtime, banks), metas
    for b in banks:
        b.close()


def _host(meta, layer: int, experts) -> BankHost:
    from vllm_nvfp4_cuda import synthetic

    host = BankHost(E, H, I, meta.router_bf16.numpy().view(np.uint16), meta.shared_gate_bf16.numpy().view(np.uint16))
    for e in experts:
        for p in range(3):
            packed, scales, div = synthetic.synthetic_expert_projection(int(e), p, H, I, SEED, layer=101 + layer)
            host.projections[p][int(e)] = QuantizedMatrix(packed.cpu().numpy(), scales.cpu().numpy(), div)
    return host


@pytest.mark.parametrize("T", [1, 64])
def test_full_shape_stack_layer_by_layer(cuda_runtime, full_stack, T):
    import torch

    from vllm_nvfp4_cuda import synthetic

    stack, metas = full_stack
    x = synthetic.synthetic_tokens(T, H, 4242 + T)
    ones = torch.ones(H, dtype=torch.bfloat16, device="cuda")

    # Per-layer synchronised calls; each layer's input, normalised input,
    # output and routing record.
    states, normed, routes = [x.clone()], [], []
    for bank in stack.banks:
        h = states[-1]
        out = torch.empty_like(h)
        bank.forward(h, residual=h, out=out, pre_norm=True)
        torch.cuda.synchronize()
        routes.append(bank.last_routing(T).ids.copy())
        normed.append(cuda_runtime.rmsnorm_bf16(h, ones).float().cpu().numpy())
        torch.cuda.synchronize()
        states.append(out)

    # The captured step replays to the synchronised result bit for bit.
    g = stack.capture(T)
    try:
        replayed = g.run(x)
        torch.cuda.synchronize()
        assert torch.equal(replayed, states[-1])
    finally:
        g.close()

    for layer in range(LAYERS):
        h_in = states[layer].float().cpu().numpy()
        router_all = np.concatenate([metas[layer].router_bf16.numpy().view(np.uint16),
                                     metas[layer].shared_gate_bf16.numpy().view(np.uint16)[None]], axis=0)
        ids, _, _ = cpu_oracle.route(router_all, normed[layer])
        np.testing.assert_array_equal(routes[layer], ids, err_msg=f"layer {layer}")
        host = _host(metas[layer], layer, sorted(set(ids[:, :8].reshape(-1).tolist()) | {E}))
        ref = moe_layer(host, normed[layer], h_in)
        got = states[layer + 1].float().cpu().numpy()
        assert rel_rmse(got, ref.out) <= REL_RMSE_TOL, layer
        assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL, layer
        del host
