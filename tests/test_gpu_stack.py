"""Resident layer stack (h <- h + MoE(RMSNorm(h)) per layer, attention
omitted) against the oracle's composition, and its CUDA-graph replay
(needs an sm_100a GPU).

* The pointer RMSNorm matches the oracle restatement within one BF16 step
  (the kernel's rsqrtf is within 2 ulp of 1/sqrt).
* Three layers of small banks at one token (in-register GEMVs) and five
  (tensor-core GEMVs) match ``moe_stack`` at the BASELINE tolerance.
* The fused pre-norm (NVFP4_MOE_PRE_NORM) gives the same bits as the
  standalone RMSNorm followed by the plain forward, on the decode path and
  on the prefill path.
* A captured step replays to the same bits as the eager stack.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import bf16_bits_from_f32, max_abs_rel, moe_stack, rel_rmse, rmsnorm_bf16

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

LAYERS = 3


@pytest.fixture(scope="module")
def stack_hosts():
    return [synthetic_np.make_bank(32, 512, 256, 700 + layer) for layer in range(LAYERS)]


@pytest.fixture(scope="module")
def stack(cuda_runtime, stack_hosts):
    from vllm_nvfp4_cuda.stack import MoeStack

    banks = [upload_bank(cuda_runtime, h) for h in stack_hosts]
    yield MoeStack(cuda_runtime, banks)
    for b in banks:
        b.close()


@pytest.mark.parametrize("rows,cols", [(1, 2048), (5, 512), (3, 1000)])
def test_rmsnorm_ptr_matches_oracle(cuda_runtime, rows, cols):
    import torch

    rng = np.random.default_rng(rows * 7 + cols)
    xbits = synthetic_np.tokens_bf16(rows, cols, rows + cols)
    wbits = bf16_bits_from_f32((rng.standard_normal(cols) * 0.5 + 1.0).astype(np.float32))
    out = cuda_runtime.rmsnorm_bf16(bits_to_bf16_tensor(xbits.reshape(rows, cols)), bits_to_bf16_tensor(wbits),
                                    1e-6)
    torch.cuda.synchronize()
    got = bf16_tensor_to_f32(out)
    ref = rmsnorm_bf16(synthetic_np.bf16_bits_to_f32(xbits).reshape(rows, cols),
                       synthetic_np.bf16_bits_to_f32(wbits), 1e-6)
    diff = np.abs(got - ref)
    assert np.all(diff <= np.abs(ref) * 2.0 ** -7 + 1e-30)
    assert np.count_nonzero(diff) <= max(2, ref.size // 1000)


@pytest.mark.parametrize("T", [1, 5])
def test_stack_matches_oracle(cuda_runtime, stack, stack_hosts, T):
    import torch

    xbits = synthetic_np.tokens_bf16(T, 512, 900 + T)
    got = stack.forward(bits_to_bf16_tensor(xbits))
    torch.cuda.synchronize()
    got = bf16_tensor_to_f32(got)
    ref = moe_stack(stack_hosts, synthetic_np.bf16_bits_to_f32(xbits))
    assert rel_rmse(got, ref) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref) <= MAX_ABS_REL_TOL


@pytest.mark.parametrize("T", [1, 5, 40, 80])
def test_fused_norm_matches_separate_norm(cuda_runtime, stack, stack_hosts, T):
    """The RMSNorm fused into the layer (routing kernel up to 64 tokens, a
    slice pre-pass above) gives the bits of the standalone RMSNorm + forward."""
    import torch

    from vllm_nvfp4_cuda.stack import MoeStack

    unfused = MoeStack(cuda_runtime, stack.banks, fused_norm=False)
    x = bits_to_bf16_tensor(synthetic_np.tokens_bf16(T, 512, 950 + T))
    a = stack.forward(x)
    b = unfused.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [1, 2])
def test_stack_graph_replay(cuda_runtime, stack, T):
    import torch

    g = stack.capture(T)
    try:
        for seed in (31, 32):
            x = bits_to_bf16_tensor(synthetic_np.tokens_bf16(T, 512, seed))
            eager = stack.forward(x)
            replayed = g.run(x)
            torch.cuda.synchronize()
            assert torch.equal(eager, replayed)
    finally:
        g.close()
