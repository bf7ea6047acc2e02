"""Oracle pinned against the reference's own Python oracle functions
(golden vectors from tests/golden/make_golden.py) and against the C port."""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import cpu_oracle, synthetic_np
from oracle.nvfp4_oracle import (
    E2M1,
    BankHost,
    bf16_bits_from_f32,
    bf16_bits_to_f32,
    decode_e4m3_scale,
    dequantize,
    dispatch,
    e2m1_encode_rne,
    e4m3_encode_rne,
    expert_forward,
    max_abs_rel,
    moe_layer,
    moe_stack,
    nvfp4_gemv,
    quantize_nvfp4,
    rel_rmse,
    rmsnorm_bf16,
    router_logits,
    top8_route,
)

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def test_decode_tables_match_reference():
    g = load("golden_decode.npz")
    np.testing.assert_array_equal(decode_e4m3_scale(np.arange(256, dtype=np.uint8)), g["e4m3"])
    np.testing.assert_array_equal(E2M1, g["e2m1"])


@pytest.mark.parametrize("case", range(4))
def test_gemv_matches_reference(case):
    g = load("golden_gemv.npz")
    packed, scales, x, div, ref = (g[f"{k}{case}"] for k in ("packed", "scales", "x", "divisor", "out"))
    out = nvfp4_gemv(packed, scales, x, float(div))
    np.testing.assert_allclose(out, ref, rtol=1e-6, atol=1e-6 * float(np.max(np.abs(ref))))
    # The C restatement of the NEON row kernel, at the reference's own GEMV gate.
    port = cpu_oracle.cpu_gemv(packed, scales, x, float(div), threads=2)
    np.testing.assert_allclose(port, ref, rtol=2e-5, atol=2e-5 * float(np.max(np.abs(ref))))
    # Dequantise-then-matmul agrees too.
    dense = dequantize(packed, scales, float(div)).astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(dense, ref, rtol=1e-5, atol=1e-5 * float(np.max(np.abs(ref))))


def test_route_matches_reference():
    g = load("golden_route.npz")
    ids, weights = top8_route(g["logits"])
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(weights, g["weights"], rtol=2e-6, atol=1e-7)


def test_route_ties_take_lowest_id():
    logits = np.zeros((3, 16), dtype=np.float32)
    logits[1, [3, 9, 12]] = 1.0
    logits[2] = np.float32(-1.0)
    logits[2, [15, 2]] = np.float32(-0.5)
    ids, weights = top8_route(logits)
    np.testing.assert_array_equal(ids[0], np.arange(8))
    np.testing.assert_array_equal(ids[1], [3, 9, 12, 0, 1, 2, 4, 5])
    np.testing.assert_array_equal(ids[2], [2, 15, 0, 1, 3, 4, 5, 6])
    np.testing.assert_allclose(weights.sum(axis=1), 1.0, rtol=1e-6)
    # -0.0 and +0.0 are equal logits: the lower id wins.
    z = np.zeros((1, 16), dtype=np.float32)
    z[0, 5] = np.float32(-0.0)
    z[0, :5] = -1
    ids, _ = top8_route(z)
    assert ids[0, 0] == 5


def test_expert_matches_reference():
    g = load("golden_expert.npz")
    H, I = 256, 128
    from oracle.nvfp4_oracle import QuantizedMatrix

    bank = BankHost(0, H, I, np.zeros((0, H), np.uint16), np.zeros(H, np.uint16))
    for p in range(3):
        bank.projections[p][0] = QuantizedMatrix(g[f"packed{p}"], g[f"scales{p}"], float(g[f"divisor{p}"]))
    out = expert_forward(bank, 0, g["x"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-4 * float(np.max(np.abs(g["out"]))))


def _sha(q):
    h = hashlib.sha256()
    for p in q:
        h.update(np.ascontiguousarray(p.packed).tobytes())
        h.update(np.ascontiguousarray(p.scales).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name", ["small", "config0"])
def test_layer_matches_reference(name):
    g = load("golden_layer.npz")
    E, H, I, seed, T = (int(v) for v in g[f"{name}_shape"])
    ids_ref = g[f"{name}_ids"]
    needed = sorted(set(int(e) for e in ids_ref.reshape(-1)) | {E})
    bank = synthetic_np.make_bank(E, H, I, seed, which=needed)
    # Generator drift guard.
    hashes = dict(h.split(":", 1) for h in g[f"{name}_hashes"].tolist())
    for e in needed:
        assert _sha([bank.projections[p][e] for p in range(3)]) == hashes[str(e)]
    x = synthetic_np.tokens_f32(T, H, seed)
    res = moe_layer(bank, x)
    np.testing.assert_array_equal(res.ids[:, :8], ids_ref)
    np.testing.assert_allclose(res.weights[:, :8], g[f"{name}_weights"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(res.logits[:, E], g[f"{name}_shared_logit"], rtol=1e-5, atol=1e-5)
    ref = g[f"{name}_out"]
    # The reference's own bank gate (bench_moe_device_bank.py:152): 1e-4.
    np.testing.assert_allclose(res.out, ref, rtol=1e-4, atol=1e-4)
    assert rel_rmse(res.out, ref) < 1e-5


def test_router_logits_bit_exact_between_numpy_and_c_port():
    bank = synthetic_np.make_bank(16, 256, 128, 3)
    dense = cpu_oracle.DenseBank.from_host(bank)
    x = synthetic_np.tokens_f32(5, 256, 3)
    _, _, _, logits_c = dense.forward(x, threads=2)
    logits_np = router_logits(bank.router_all(), x)
    np.testing.assert_array_equal(logits_np.view(np.uint32), logits_c.view(np.uint32))
    exact = bf16_bits_to_f32(bank.router_all()).astype(np.float64) @ x.astype(np.float64).T
    np.testing.assert_allclose(logits_np, exact.T, rtol=1e-5, atol=2e-5)


def test_c_route_matches_numpy_oracle_with_ties_and_bias():
    """The C routing entry (the full-size prefill checker) against
    moe_layer's routing: logits bit for bit, ids exactly, on a skewed bank
    with duplicated router rows and an all-zero token (every logit ties)."""
    bank = synthetic_np.make_bank(64, 256, 128, 9, which=[], skew=True)
    w = bf16_bits_to_f32(bank.router_bf16).copy()
    w[7] = w[30] = w[2]
    bank.router_bf16 = bf16_bits_from_f32(w)
    bank.router_bias[[2, 7, 30]] = np.float32(0.5)
    x = synthetic_np.tokens_f32(40, 256, 9)
    x[0] = 0.0
    ids, weights, logits = cpu_oracle.route(bank.router_all(), x, bank.router_bias, threads=3)
    ref = router_logits(bank.router_all(), x)
    ref[:, :64] = (ref[:, :64] + bank.router_bias).astype(np.float32)
    np.testing.assert_array_equal(logits.view(np.uint32), ref.view(np.uint32))
    top, tw = top8_route(ref[:, :64])
    np.testing.assert_array_equal(ids[:, :8], top)
    np.testing.assert_allclose(weights[:, :8], tw, rtol=2e-6, atol=1e-7)
    assert (ids[:, 8] == 64).all()
    assert list(ids[0, :3]) == [2, 7, 30]


def test_c_port_layer_matches_numpy_oracle():
    bank = synthetic_np.make_bank(16, 256, 128, 5, skew=True)
    dense = cpu_oracle.DenseBank.from_host(bank)
    x = synthetic_np.tokens_f32(6, 256, 5)
    residual = synthetic_np.tokens_f32(6, 256, 6)
    out, ids, weights, _ = dense.forward(x, residual, threads=3)
    ref = moe_layer(bank, x, residual)
    np.testing.assert_array_equal(ids, ref.ids)
    np.testing.assert_allclose(weights, ref.weights, rtol=1e-5, atol=1e-7)
    assert rel_rmse(out, ref.out) < 1e-5
    assert max_abs_rel(out, ref.out) < 1e-4


def test_dispatch_permutation_is_stable_and_grouped():
    rng = np.random.default_rng(1)
    T, E = 37, 32
    ids = np.stack([rng.choice(E, 8, replace=False) for _ in range(T)]).astype(np.int32)
    counts, offsets, perm = dispatch(ids, E)
    assert counts.sum() == T * 8 and offsets[-1] == T * 8
    np.testing.assert_array_equal(counts, np.bincount(ids.reshape(-1), minlength=E))
    flat = ids.reshape(-1)
    for e in range(E):
        seg = perm[offsets[e] : offsets[e + 1]]
        assert np.all(flat[seg] == e)
        assert np.all(np.diff(seg // 8) > 0)  # tokens ascending, each once
    # Edge cases: a single token and experts that receive nothing.
    c1, o1, p1 = dispatch(np.arange(8, dtype=np.int32)[None], 256)
    assert c1[:8].tolist() == [1] * 8 and c1[8:].sum() == 0 and p1.tolist() == list(range(8))


def test_quantizer_roundtrip_and_rules():
    rng = np.random.default_rng(2)
    w = rng.standard_normal((64, 256)).astype(np.float32) * np.float32(0.02)
    q = quantize_nvfp4(w)
    deq = dequantize(q.packed, q.scales, q.global_scale)
    # Re-quantising the dequantised tensor reproduces the same codes and scales.
    q2 = quantize_nvfp4(deq)
    np.testing.assert_array_equal(q2.scales, q.scales)
    np.testing.assert_array_equal(q2.packed, q.packed)
    assert rel_rmse(deq, w) < 0.15
    # E2M1 ties go to the even code; saturation at 6.
    vals = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.25, -0.0], dtype=np.float32)
    assert e2m1_encode_rne(vals).tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 8, 8]
    # E4M3: exact values map to themselves, 448 saturates, ties to even.
    assert e4m3_encode_rne(np.array([448.0, 1000.0, 1.0, 2.0**-9, 1.0625, 1.1875])).tolist() == [
        0x7E, 0x7E, 0x38, 0x01, 0x38, 0x3A]
    # All-zero tensor.
    z = quantize_nvfp4(np.zeros((16, 32), dtype=np.float32))
    assert not z.packed.any() and not z.scales.any()


def test_torch_quantizer_matches_oracle_quantizer():
    torch = pytest.importorskip("torch")
    from vllm_nvfp4_cuda.synthetic import quantize_nvfp4 as quant_torch

    rng = np.random.default_rng(4)
    for shape, scale in [((64, 256), 0.02), ((32, 512), 3.0), ((16, 128), 1e-4)]:
        w = (rng.standard_normal(shape) * scale).astype(np.float32)
        w[0, :16] = 0.0
        w[1, 3] = np.float32(0.0) * -1
        q = quantize_nvfp4(w)
        packed, scales, divisor = quant_torch(torch.from_numpy(w))
        np.testing.assert_array_equal(packed.numpy(), q.packed)
        np.testing.assert_array_equal(scales.numpy(), q.scales)
        assert np.float32(divisor) == np.float32(q.global_scale)
    # E4M3 rounding of torch's float8 cast equals the oracle's on a sweep.
    v = np.concatenate([np.linspace(0, 460, 20001), np.exp2(np.linspace(-12, 9, 4001))]).astype(np.float32)
    t = torch.from_numpy(np.minimum(v, 448.0)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(t, e4m3_encode_rne(v))


def test_bf16_roundtrip():
    x = np.array([1.0, -2.5, 1.00390625, 3.4e38, 1e-40], dtype=np.float32)
    b = bf16_bits_from_f32(x)
    assert bf16_bits_to_f32(b)[0] == 1.0 and bf16_bits_to_f32(b)[1] == -2.5


def test_rmsnorm_restatement():
    """The oracle's RMSNorm (CUDA kernel's reduction order, BF16 output) is
    the lab's x * rsqrt(mean(x^2) + eps) * w to within one BF16 rounding."""
    rng = np.random.default_rng(5)
    x = bf16_bits_to_f32(bf16_bits_from_f32(rng.standard_normal((4, 2048)).astype(np.float32) * 3))
    w = bf16_bits_to_f32(bf16_bits_from_f32(rng.standard_normal(2048).astype(np.float32) * 0.5 + 1))
    exact = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * w
    got = rmsnorm_bf16(x, w, 1e-6)
    assert np.all(np.abs(got - exact) <= np.abs(exact) * 2.0 ** -8 + 1e-12)
    np.testing.assert_array_equal(bf16_bits_to_f32(bf16_bits_from_f32(got)), got)


def test_stack_composes_layers():
    """moe_stack is h <- BF16(h + moe_layer(RMSNorm(h))) layer by layer."""
    banks = [synthetic_np.make_bank(8, 128, 64, 40 + i) for i in range(2)]
    x = bf16_bits_to_f32(synthetic_np.tokens_bf16(2, 128, 3))
    h = x
    for b in banks:
        h = bf16_bits_to_f32(bf16_bits_from_f32(moe_layer(b, rmsnorm_bf16(h), h).out))
    np.testing.assert_array_equal(moe_stack(banks, x), h)
