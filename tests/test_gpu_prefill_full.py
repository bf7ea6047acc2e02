"""Prefill at the BASELINE shapes against the CPU oracle (needs an sm_100a GPU).

Config 2: E 256, H 2048, I 512 (the full 257-expert bank), 4096 tokens,
near-uniform router. Config 3: the same bank shape with the skew bias
b_e = 2 log(1 / rank_e^1.2), 8192 tokens, where the hottest expert receives
every token (its group spans 64 GEMM column tiles).

* Routing of EVERY token is compared with the C restatement
  (``oracle.cpu_oracle.route``: the FP32 fixed-order logits and the
  lowest-id top-8 of ``oracle.nvfp4_oracle.moe_layer``): ids, counts and the
  dispatch permutation bit-exact, weights to 2e-6. The prefill kernels pick
  candidates from approximate tensor-core logits and re-check them exactly, so
  this is the check that no 8th/9th pick flips at full size.
* Outputs of a seeded sample of 256+ tokens (including tokens routed to the
  hottest expert, spread over its column tiles, and the first and last
  token) are compared with the FP32 dequantise-then-matmul oracle
  ``moe_layer`` at the BASELINE bound (relative RMSE <= 2e-3,
  max-abs-relative <= 1e-2) and with the same-terms oracle
  ``moe_layer_prefill`` at the default (4, 3) activation terms, rounded to
  BF16 like the GPU output (relative RMSE <= 1e-3). The call is made twice:
  without a residual, so the bound measures the layer's own error rather
  than the BF16 rounding of a residual ~5x larger than the layer output, and
  with the residual the BASELINE configs name.

Every token's output depends only on that token, so the sampled oracle rows
are the full call's rows.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cpu_oracle, synthetic_np
from oracle.nvfp4_oracle import (BankHost, QuantizedMatrix, bf16_bits_from_f32, dispatch, max_abs_rel, moe_layer,
                                 moe_layer_prefill, rel_rmse)

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL

pytestmark = pytest.mark.gpu

E, H, I = 256, 2048, 512
SAME_TERMS_TOL = 1e-3
SAMPLE = 224


def _bf16(v: np.ndarray) -> np.ndarray:
    return synthetic_np.bf16_bits_to_f32(bf16_bits_from_f32(np.asarray(v, dtype=np.float32)))


def _sample(ids: np.ndarray, counts: np.ndarray, T: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    picked = set(rng.choice(T, SAMPLE, replace=False).tolist())
    hot = int(np.argmax(counts))
    hot_tokens = np.nonzero((ids[:, :8] == hot).any(axis=1))[0]
    step = max(1, len(hot_tokens) // 32)
    picked.update(hot_tokens[::step][:32].tolist())
    picked.update([0, T - 1])
    return np.asarray(sorted(picked), dtype=np.int64)


def _host_for(meta, experts, seed) -> BankHost:
    from vllm_nvfp4_cuda import synthetic

    host = BankHost(E, H, I, meta.router_bf16.numpy().view(np.uint16), meta.shared_gate_bf16.numpy().view(np.uint16))
    if meta.router_bias is not None:
        host.router_bias = meta.router_bias.numpy().astype(np.float32)
    for e in experts:
        for p in range(3):
            packed, scales, div = synthetic.synthetic_expert_projection(int(e), p, H, I, seed)
            host.projections[p][int(e)] = QuantizedMatrix(packed.cpu().numpy(), scales.cpu().numpy(), div)
    return host


@pytest.mark.parametrize("config", ["config2_uniform_4096", "config3_skewed_8192"])
def test_prefill_full_shape(cuda_runtime, config):
    import torch

    from vllm_nvfp4_cuda import synthetic

    skew = config.startswith("config3")
    T = 8192 if skew else 4096
    seed = 0
    bank, meta = synthetic.build_bank(cuda_runtime, E, H, I, seed, skew=skew)
    try:
        x = synthetic.synthetic_tokens(T, H, seed + 11)
        r = synthetic.synthetic_tokens(T, H, seed + 12)
        bare = bank.forward(x)
        torch.cuda.synchronize()
        bare_all = bare.float().cpu().numpy()
        out = bank.forward(x, residual=r)
        torch.cuda.synchronize()
        routing = bank.last_routing(T)
        got_all = out.float().cpu().numpy()
    finally:
        bank.close()
    xf = x.float().cpu().numpy()
    rf = r.float().cpu().numpy()
    router_all = np.concatenate([meta.router_bf16.numpy().view(np.uint16),
                                 meta.shared_gate_bf16.numpy().view(np.uint16)[None]], axis=0)
    bias = None if meta.router_bias is None else meta.router_bias.numpy()
    ids, weights, _ = cpu_oracle.route(router_all, xf, bias)
    counts, _, perm = dispatch(ids[:, :8], E)

    # Routing of every token.
    np.testing.assert_array_equal(routing.ids, ids)
    np.testing.assert_allclose(routing.weights, weights, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(routing.counts, counts)
    np.testing.assert_array_equal(routing.perm, perm)
    if skew:
        assert counts.max() >= 8 * counts.mean(), "the skew bias must concentrate load"

    # Outputs of the sampled tokens.
    sample = _sample(ids, counts, T, seed + 5)
    experts = sorted(set(ids[sample, :8].reshape(-1).tolist()) | {E})
    host = _host_for(meta, experts, seed)
    ref = moe_layer(host, xf[sample])
    np.testing.assert_array_equal(ref.ids, ids[sample])
    got = bare_all[sample]
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    same = moe_layer_prefill(host, xf[sample], None, 4, 3)
    assert rel_rmse(got, _bf16(same.out)) <= SAME_TERMS_TOL
    # With the residual (the oracle adds it in float64 before any rounding).
    with_res = ref.out + rf[sample].astype(np.float64)
    assert rel_rmse(got_all[sample], with_res) <= REL_RMSE_TOL
    assert max_abs_rel(got_all[sample], with_res) <= MAX_ABS_REL_TOL
