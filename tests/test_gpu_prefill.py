"""Prefill path (calls above 64 tokens) vs the CPU oracle (needs an sm_100a GPU).

* The activation quantiser is compared bit for bit (codes, scale words, row
  scales) with ``oracle.nvfp4_oracle.quantize_rows_split``.
* Routing of a prefill call (approximate tensor-core logits + exact
  re-check) must equal the oracle's FP32 fixed-order routing bit for bit:
  ids, counts and the dispatch permutation.
* Layer outputs are compared with ``moe_layer_prefill`` (the same activation
  terms; tight tolerance) and, at the default 4/3 terms, with the FP32
  activation oracle ``moe_layer`` at the BASELINE tolerance (relative RMSE
  <= 2e-3, max-abs-relative <= 1e-2).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import (bf16_bits_from_f32, max_abs_rel, moe_layer, moe_layer_prefill, quantize_rows_split,
                                 rel_rmse)

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

# GPU vs the same-numerics oracle rounded to BF16 like the GPU output: FP32
# tensor-core accumulation order, FP16 partials and rare act-code flips only.
SAME_TERMS_TOL = 1e-3


def _bf16(v: np.ndarray) -> np.ndarray:
    return synthetic_np.bf16_bits_to_f32(bf16_bits_from_f32(np.asarray(v, dtype=np.float32)))


def _rows(rows: int, cols: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[0] = 0.0                                  # all-zero row: g = 1, every code 0
    x[1] *= np.float32(1e-3)                    # small magnitudes
    x[2, :16] = np.float32(448.0 * 6.0)         # a saturating block
    x[3, ::7] = 0.0                             # zeros inside blocks (signed zero canonicalisation)
    x[4] = -np.abs(x[4]) * np.float32(1e-6)     # tiny negatives that round to zero
    return x


@pytest.mark.parametrize("terms", [1, 2, 3, 4])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_quantize_rows_bit_exact(cuda_runtime, terms, dtype):
    import torch

    rows, cols = 37, 256
    x = _rows(rows, cols, 7 + terms)
    if dtype == "bf16":
        t = torch.from_numpy(x).to(torch.bfloat16)
    else:
        t = torch.from_numpy(x).to(torch.float16)
    xf = t.to(torch.float32).numpy()
    codes, words, g = cuda_runtime.quantize_rows(t.cuda(), terms)
    torch.cuda.synchronize()
    ref = quantize_rows_split(xf, terms)
    np.testing.assert_array_equal(g.cpu().numpy().view(np.uint32), ref.g.view(np.uint32))
    np.testing.assert_array_equal(words.cpu().numpy().view(np.uint32), ref.words)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref.codes)


@pytest.fixture(scope="module")
def prefill_host():
    # Multiples of 256 (the prefill GEMM tiles); 32 experts keep the oracle quick.
    return synthetic_np.make_bank(32, 512, 256, 91)


@pytest.fixture(scope="module")
def prefill_bank(cuda_runtime, prefill_host):
    bank = upload_bank(cuda_runtime, prefill_host)
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


@pytest.mark.parametrize("T", [65, 200, 513])
def test_prefill_default_terms(cuda_runtime, prefill_bank, prefill_host, T):
    got, xf, rf = _run(prefill_bank, prefill_host, T, 300 + T)
    same = moe_layer_prefill(prefill_host, xf, rf, 4, 3)
    _check_routing(prefill_bank, same, T)
    assert rel_rmse(got, _bf16(same.out)) <= SAME_TERMS_TOL
    fp32 = moe_layer(prefill_host, xf, rf)
    assert rel_rmse(got, fp32.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, fp32.out) <= MAX_ABS_REL_TOL


@pytest.mark.parametrize("terms", [(1, 1), (2, 2), (3, 3)])
def test_prefill_terms(cuda_runtime, prefill_bank, prefill_host, terms):
    T = 160
    prefill_bank.set_prefill_terms(*terms)
    try:
        got, xf, _ = _run(prefill_bank, prefill_host, T, 700 + terms[0], residual=False)
    finally:
        prefill_bank.set_prefill_terms(4, 3)
    same = moe_layer_prefill(prefill_host, xf, None, *terms)
    assert rel_rmse(got, _bf16(same.out)) <= SAME_TERMS_TOL


def test_prefill_skewed_routing(cuda_runtime):
    host = synthetic_np.make_bank(64, 256, 256, 93, skew=True)
    bank = upload_bank(cuda_runtime, host)
    T = 300
    got, xf, rf = _run(bank, host, T, 900)
    ref = moe_layer(host, xf, rf)
    _check_routing(bank, ref, T)
    # Skew concentrates load: the hottest expert spans several column tiles.
    assert ref.counts.max() > 128
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    bank.close()
