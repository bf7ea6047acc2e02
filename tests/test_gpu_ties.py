"""Routing ties on the GPU: the lab's selection keeps the LOWEST expert id among
equal logits (``candidate > best || (candidate == best && expert < best_id)``,
native_nvfp4/kernels/nvfp4_gemv.cl:1271-1275). Needs an sm_100a GPU.

Exact ties are made three ways, each giving bit-identical FP32 logits on
every implementation:

* duplicated router rows: rows {3, 17, 40, 41} are 4x row 3 and rows
  {50, 51, 52} are -4x row 3 (scaling by a power of two and negating are
  exact in BF16), so for most tokens one of the two groups holds the largest
  logits, all equal within the group; rows {5, 6} are 2x row 5;
* equal router biases on zero rows: row 10 is all -0 (BF16 0x8000), row 11
  all +0, both with bias 5.0, so both logits are exactly 5.0 for any token;
* an all-zero token and an all -0 token: every logit is +0 plus its bias,
  so 50+ experts tie at 0 and the picks after the biased ones must be the
  lowest ids in order. At 256 experts this sends the prefill selection past
  its 64-candidate list into its streaming fallback.

A +0/-0 pair of LOGITS cannot arise: every logit is a fixed-order FP32 sum
that starts from +0, and in round-to-nearest x + (-0) = x and a + (-a) = +0,
so -0 products (row 10, the -0 token) and exact cancellations all give +0.
The -0 router row and the -0 token exercise exactly that; the tensor-core
approximate logits of the prefill path may hold -0, which its candidate
selection treats as +0.

Ids, counts and the dispatch permutation are compared bit-exactly with the
oracle, through every decode variant (T 1, 4, 32; the fused one-token
kernel at T 1) and the prefill path (T 65, 200); outputs within the
BASELINE bound.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cpu_oracle, synthetic_np
from oracle.nvfp4_oracle import bf16_bits_from_f32, bf16_bits_to_f32, max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

TIE_GROUPS = ((3, 17, 40, 41), (5, 6), (50, 51, 52))


def _tie_host(experts: int, hidden: int, seed: int):
    host = synthetic_np.make_bank(experts, hidden, 256, seed)
    w = bf16_bits_to_f32(host.router_bf16).copy()
    for e in (17, 40, 41):
        w[e] = np.float32(4.0) * w[3]
    w[3] = np.float32(4.0) * w[3]
    for e in (50, 51, 52):
        w[e] = -w[3]
    w[5] = np.float32(2.0) * w[5]
    w[6] = w[5]
    router = bf16_bits_from_f32(w)
    router[10] = 0x8000
    router[11] = 0x0000
    host.router_bf16 = np.ascontiguousarray(router)
    bias = np.zeros(experts, dtype=np.float32)
    bias[10] = bias[11] = np.float32(5.0)
    host.router_bias = bias
    return host


def _tokens(T: int, hidden: int, seed: int) -> np.ndarray:
    bits = synthetic_np.tokens_bf16(T, hidden, seed)
    bits[0] = 0x0000
    if T > 1:
        bits[1] = 0x8000
    return np.ascontiguousarray(bits)


@pytest.fixture(scope="module")
def tie_host64():
    return _tie_host(64, 512, 41)


@pytest.fixture(scope="module")
def tie_bank64(cuda_runtime, tie_host64):
    bank = upload_bank(cuda_runtime, tie_host64)
    yield bank
    bank.close()


@pytest.fixture(scope="module")
def tie_host256():
    return _tie_host(256, 256, 43)


@pytest.fixture(scope="module")
def tie_bank256(cuda_runtime, tie_host256):
    bank = upload_bank(cuda_runtime, tie_host256)
    yield bank
    bank.close()


def _check(bank, host, T, seed):
    import torch

    xbits = _tokens(T, host.hidden, seed)
    out = bank.forward(bits_to_bf16_tensor(xbits))
    torch.cuda.synchronize()
    xf = synthetic_np.bf16_bits_to_f32(xbits)
    ref = moe_layer(host, xf)
    r = bank.last_routing(T)
    np.testing.assert_array_equal(r.ids, ref.ids)
    np.testing.assert_allclose(r.weights, ref.weights, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(r.counts, ref.counts)
    np.testing.assert_array_equal(r.perm, ref.perm)
    # The C restatement agrees (its own selection loop: strict >, ids ascending).
    c_ids, _, _ = cpu_oracle.route(host.router_all(), xf, host.router_bias)
    np.testing.assert_array_equal(c_ids, ref.ids)
    got = bf16_tensor_to_f32(out)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    return ref


def _assert_ties_present(ref, experts):
    ids = ref.ids[:, :8]
    # The zero token: the two biased experts (10 before 11), then ids 0, 1, ...
    zero_expect = [10, 11] + [e for e in range(experts) if e not in (10, 11)][:6]
    np.testing.assert_array_equal(ids[0], zero_expect)
    # Wherever tied experts are picked they come lowest id first, and most
    # tokens pick a whole duplicated group.
    whole = 0
    for row in ids[2:]:
        for g in TIE_GROUPS:
            pos = [list(row).index(e) for e in g if e in row]
            assert pos == sorted(pos), (row, g)
            whole += len(pos) == len(g) and len(g) > 2
    assert whole >= (len(ids) - 2) // 3, whole


@pytest.mark.parametrize("kernels", ["tensor_core", "in_register", "fused_token"])
@pytest.mark.parametrize("T", [1, 4, 32, 48])
def test_decode_ties(cuda_runtime, tie_bank64, tie_host64, kernels, T):
    tie_bank64.set_decode_kernels(kernels)
    try:
        ref = _check(tie_bank64, tie_host64, T, 500 + T)
    finally:
        tie_bank64.set_decode_kernels("tensor_core")
    if T >= 4:
        _assert_ties_present(ref, tie_host64.experts)


@pytest.mark.parametrize("T", [65, 200])
def test_prefill_ties(cuda_runtime, tie_bank64, tie_host64, T):
    ref = _check(tie_bank64, tie_host64, T, 600 + T)
    _assert_ties_present(ref, tie_host64.experts)


@pytest.mark.parametrize("T", [1, 32, 64, 65])
def test_ties_256_experts(cuda_runtime, tie_bank256, tie_host256, T):
    """256 experts: the zero token ties 254 logits at 0, beyond the prefill
    selection's 64-candidate list (its streaming fallback)."""
    ref = _check(tie_bank256, tie_host256, T, 700 + T)
    if T >= 4:
        _assert_ties_present(ref, tie_host256.experts)
