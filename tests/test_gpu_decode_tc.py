"""Decode expert GEMVs: the tensor-core variant (tcgen05 block-scaled MMA,
four NVFP4 activation terms per row) against the oracle, and the
in-register variant selected through ``set_decode_kernels`` (needs an
sm_100a GPU).

* The tensor-core variant computes the same arithmetic as the oracle's
  ``moe_layer_prefill`` at (4, 4) terms; outputs must agree with it rounded
  to BF16 (FP32 tensor-core accumulation order and FP16 activations only)
  and with the FP32 oracle ``moe_layer`` at the BASELINE tolerance.
* Routing (ids, counts, dispatch permutation) is bit-exact in both variants.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import bf16_bits_from_f32, max_abs_rel, moe_layer, moe_layer_prefill, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

SAME_TERMS_TOL = 1e-3


def _bf16(v: np.ndarray) -> np.ndarray:
    return synthetic_np.bf16_bits_to_f32(bf16_bits_from_f32(np.asarray(v, dtype=np.float32)))


@pytest.fixture(scope="module")
def tc_host():
    # H and I multiples of 256 (the tensor-core tiles); 32 experts keep the oracle quick.
    return synthetic_np.make_bank(32, 512, 256, 61)


@pytest.fixture(scope="module")
def tc_bank(cuda_runtime, tc_host):
    bank = upload_bank(cuda_runtime, tc_host)
    yield bank
    bank.close()


def _run(bank, host, T, seed, residual=True):
    import torch

    H = host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, seed)
    rbits = synthetic_np.tokens_bf16(T, H, seed + 1) if residual else None
    out = bank.forward(bits_to_bf16_tensor(xbits), residual=bits_to_bf16_tensor(rbits) if residual else None)
    torch.cuda.synchronize()
    xf = synthetic_np.bf16_bits_to_f32(xbits)
    rf = synthetic_np.bf16_bits_to_f32(rbits) if residual else None
    return bf16_tensor_to_f32(out), xf, rf


def _check_routing(bank, ref, T):
    r = bank.last_routing(T)
    np.testing.assert_array_equal(r.ids, ref.ids)
    np.testing.assert_allclose(r.weights, ref.weights, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(r.counts, ref.counts)
    np.testing.assert_array_equal(r.perm, ref.perm)


# Above 32 tokens each expert's tokens split into two groups by token half
# (tokens 0-31 and 32-63), each a 128-row tile of terms.
@pytest.mark.parametrize("T", [4, 5, 12, 17, 32, 33, 40, 63, 64])
def test_tensor_core_decode(cuda_runtime, tc_bank, tc_host, T):
    got, xf, rf = _run(tc_bank, tc_host, T, 400 + T)
    same = moe_layer_prefill(tc_host, xf, rf, 4, 4)
    _check_routing(tc_bank, same, T)
    assert rel_rmse(got, _bf16(same.out)) <= SAME_TERMS_TOL
    fp32 = moe_layer(tc_host, xf, rf)
    assert rel_rmse(got, fp32.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, fp32.out) <= MAX_ABS_REL_TOL


def test_f32_abi_one_token(cuda_runtime, tc_bank, tc_host):
    """The reference ABI (FP32 x, FP32 out, one token): in-register variant at one token."""
    H = tc_host.hidden
    x = (synthetic_np.tokens_f32(1, H, 77) * np.float32(0.2)).astype(np.float32)
    xb = cuda_runtime.upload_buffer(np.ascontiguousarray(x[0]))
    out = cuda_runtime.create_buffer(H * 4)
    tc_bank.decode_device(xb, out)
    cuda_runtime.synchronize()
    got = out.download((1, H))
    fp32 = moe_layer(tc_host, x)
    assert rel_rmse(got, fp32.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, fp32.out) <= MAX_ABS_REL_TOL


@pytest.mark.parametrize("T", [1, 3, 8, 32, 48])
def test_in_register_decode(cuda_runtime, tc_bank, tc_host, T):
    tc_bank.set_decode_kernels("in_register")
    try:
        got, xf, rf = _run(tc_bank, tc_host, T, 500 + T)
    finally:
        tc_bank.set_decode_kernels("tensor_core")
    ref = moe_layer(tc_host, xf, rf)
    _check_routing(tc_bank, ref, T)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL


@pytest.mark.parametrize("T", [16, 48])
def test_variants_alternate(cuda_runtime, tc_bank, tc_host, T):
    """Switching variants between calls leaves no stale state behind."""
    outs = []
    for kind in ("tensor_core", "in_register", "tensor_core"):
        tc_bank.set_decode_kernels(kind)
        got, xf, rf = _run(tc_bank, tc_host, T, 600)
        outs.append(got)
    tc_bank.set_decode_kernels("tensor_core")
    np.testing.assert_array_equal(outs[0], outs[2])
    ref = moe_layer(tc_host, xf, rf)
    for got in outs:
        assert rel_rmse(got, ref.out) <= REL_RMSE_TOL


@pytest.mark.parametrize("T", [32, 64])
def test_tensor_core_decode_hot_expert(cuda_runtime, T):
    """Skewed routing: experts that take most of the tokens (full 128-row B
    tiles; at 64 tokens experts with more than 32 tokens, whose down
    products run as two groups, one per token half)."""
    host = synthetic_np.make_bank(64, 256, 256, 63, skew=True)
    bank = upload_bank(cuda_runtime, host)
    got, xf, rf = _run(bank, host, T, 650)
    ref = moe_layer(host, xf, rf)
    _check_routing(bank, ref, T)
    assert ref.counts.max() >= T // 2
    if T > 32:
        assert (ref.counts > 32).any()
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    bank.close()


def test_set_decode_kernels_rejects_unknown(cuda_runtime, tc_bank):
    with pytest.raises(ValueError):
        tc_bank.set_decode_kernels("bogus")
    with pytest.raises(RuntimeError):
        cuda_runtime._check(cuda_runtime.lib.nvfp4_moe_bank_set_decode_kernels(tc_bank.handle, 7),
                            "nvfp4_moe_bank_set_decode_kernels")
