"""CUDA path vs the CPU oracle, through the C ABI (needs an sm_100a GPU).

Routing ids, dispatch permutations and counts are compared bit-exactly;
router logits bit-exactly (same FP32 lane order on both sides); layer
outputs within the BASELINE tolerance: relative RMSE <= 2e-3 and
max-abs-relative <= 1e-2 against the FP32 dequantise-then-matmul oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import BankHost, QuantizedMatrix, max_abs_rel, moe_layer, rel_rmse, router_logits

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_host():
    return synthetic_np.make_bank(16, 256, 128, 21)


@pytest.fixture(scope="module")
def wide_host():
    # 256 experts (the real top-8 of 256 selection) at a reduced width.
    return synthetic_np.make_bank(256, 512, 256, 22)


@pytest.fixture(scope="module")
def small_bank(cuda_runtime, small_host):
    bank = upload_bank(cuda_runtime, small_host)
    yield bank
    bank.close()


@pytest.fixture(scope="module")
def wide_bank(cuda_runtime, wide_host):
    bank = upload_bank(cuda_runtime, wide_host)
    yield bank
    bank.close()


def check_routing(bank, ref, T):
    r = bank.last_routing(T)
    np.testing.assert_array_equal(r.ids, ref.ids)
    np.testing.assert_allclose(r.weights, ref.weights, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(r.counts, ref.counts)
    np.testing.assert_array_equal(r.perm, ref.perm)


def test_reference_decode_abi_f32(cuda_runtime, small_bank, small_host):
    rt = cuda_runtime
    H = small_host.hidden
    x = (synthetic_np.tokens_f32(1, H, 31) * np.float32(0.2)).astype(np.float32)
    xb = rt.upload_buffer(np.ascontiguousarray(x[0]))
    out = rt.create_buffer(H * 4)
    small_bank.decode_device(xb, out)
    rt.synchronize()
    got = out.download((1, H))
    ref = moe_layer(small_host, x)
    np.testing.assert_array_equal(small_bank.last_logits(1).view(np.uint32), ref.logits.view(np.uint32))
    check_routing(small_bank, ref, 1)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    xb.close()
    out.close()


@pytest.mark.parametrize("T", [1, 2, 3, 8, 9, 16, 31, 32, 33, 64])
def test_forward_bf16_batched(cuda_runtime, wide_bank, wide_host, T):
    import torch

    H = wide_host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, 100 + T)
    rbits = synthetic_np.tokens_bf16(T, H, 200 + T)
    x = bits_to_bf16_tensor(xbits)
    res = bits_to_bf16_tensor(rbits)
    out = wide_bank.forward(x, residual=res)
    torch.cuda.synchronize()
    ref = moe_layer(wide_host, synthetic_np.bf16_bits_to_f32(xbits), synthetic_np.bf16_bits_to_f32(rbits))
    logits = wide_bank.last_logits(T)
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits.view(np.uint32))
    check_routing(wide_bank, ref, T)
    got = bf16_tensor_to_f32(out)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    # Element-wise: within one BF16 rounding of the output plus the BASELINE
    # relative tolerance on the MoE contribution.
    moe_only = ref.out - synthetic_np.bf16_bits_to_f32(rbits)
    bound = np.abs(ref.out) * 2.0**-8 + MAX_ABS_REL_TOL * np.max(np.abs(moe_only))
    assert np.all(np.abs(got - ref.out) <= bound)


def test_forward_without_residual_and_buffers(cuda_runtime, small_bank, small_host):
    rt = cuda_runtime
    T, H = 5, small_host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, 41)
    xb = rt.upload_buffer(np.ascontiguousarray(xbits))
    out = rt.create_buffer(T * H * 2)
    small_bank.forward_device(xb, T, out)
    rt.synchronize()
    got = synthetic_np.bf16_bits_to_f32(out.download((T, H), np.uint16))
    ref = moe_layer(small_host, synthetic_np.bf16_bits_to_f32(xbits))
    check_routing(small_bank, ref, T)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    xb.close()
    out.close()


@pytest.mark.parametrize("T", [1, 32, 150])
def test_forward_host_matches_device_forward(cuda_runtime, wide_bank, wide_host, T):
    """nvfp4_moe_bank_forward_host_bf16 (host buffers in, host buffer out, one
    call) gives the bits of the device-pointer forward: pinned torch tensors
    and numpy arrays of BF16 bits, with and without the residual, and a
    second, smaller call after a larger one (the staging is reused)."""
    import torch

    H = wide_host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, 1100 + T)
    rbits = synthetic_np.tokens_bf16(T, H, 1200 + T)
    x, r = bits_to_bf16_tensor(xbits), bits_to_bf16_tensor(rbits)
    want = wide_bank.forward(x, residual=r)
    want_bare = wide_bank.forward(x)
    torch.cuda.synchronize()
    want = want.cpu().view(torch.int16).numpy()
    want_bare = want_bare.cpu().view(torch.int16).numpy()
    hx = torch.from_numpy(xbits.view(np.int16)).view(torch.bfloat16).pin_memory()
    hr = torch.from_numpy(rbits.view(np.int16)).view(torch.bfloat16).pin_memory()
    got = wide_bank.forward_host(hx, residual=hr)
    np.testing.assert_array_equal(got.view(torch.int16).numpy(), want)
    got_np = wide_bank.forward_host(np.ascontiguousarray(xbits))
    np.testing.assert_array_equal(got_np.view(np.int16), want_bare)
    check_routing(wide_bank, moe_layer(wide_host, synthetic_np.bf16_bits_to_f32(xbits)), T)
    want1 = wide_bank.forward(x[:1].contiguous(), residual=r[:1].contiguous())
    torch.cuda.synchronize()
    one = wide_bank.forward_host(np.ascontiguousarray(xbits[:1]), residual=np.ascontiguousarray(rbits[:1]))
    np.testing.assert_array_equal(one.view(np.int16), want1.cpu().view(torch.int16).numpy())


@pytest.mark.parametrize("T", [1, 4, 32, 48])
def test_forward_host_buffer_kinds(cuda_runtime, wide_bank, wide_host, T):
    """Decode-sized host forwards read a page-locked residual and store their
    rows into a page-locked dst over the bus; pageable buffers go through the
    device staging. Every mix gives the device forward's bits, and pinned
    buffers that are row windows of larger pinned tensors are read and
    written inside the window only."""
    import torch

    H = wide_host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, 1300 + T)
    rbits = synthetic_np.tokens_bf16(T, H, 1400 + T)
    x, r = bits_to_bf16_tensor(xbits), bits_to_bf16_tensor(rbits)
    want = wide_bank.forward(x, residual=r)
    torch.cuda.synchronize()
    want = want.cpu().view(torch.int16).numpy()
    hx = torch.from_numpy(xbits.view(np.int16)).view(torch.bfloat16).pin_memory()
    r_pageable = torch.from_numpy(rbits.view(np.int16)).view(torch.bfloat16).clone()
    r_big = torch.full((T + 5, H), -3.0, dtype=torch.bfloat16).pin_memory()
    r_big[2:2 + T] = r_pageable
    r_window = r_big[2:2 + T]
    o_pageable = torch.empty(T, H, dtype=torch.bfloat16)
    o_big = torch.full((T + 6, H), 7.0, dtype=torch.bfloat16).pin_memory()
    o_window = o_big[3:3 + T]
    assert not r_pageable.is_pinned() and not o_pageable.is_pinned()
    assert r_window.is_pinned() and o_window.is_pinned() and o_window.is_contiguous()
    for res in (r_pageable, r_window):
        for out in (o_pageable, o_window):
            out.zero_()
            wide_bank.forward_host(hx, residual=res, out=out)
            np.testing.assert_array_equal(out.view(torch.int16).numpy(), want)
    assert bool((o_big[:3] == 7.0).all()) and bool((o_big[3 + T:] == 7.0).all())
    assert bool((r_big[:2] == -3.0).all()) and bool((r_big[2 + T:] == -3.0).all())


@pytest.mark.parametrize("T", [4, 40, 100])
def test_forward_host_pre_norm(cuda_runtime, wide_bank, wide_host, T):
    """The host forward with the bank's RMSNorm applied first gives the device
    forward's bits: fused into routing (4 tokens, pinned dst written by the
    combine kernel), a separate normalisation into the staged output rows
    (40 tokens), and the prefill path (100 tokens)."""
    import torch

    H = wide_host.hidden
    g = torch.Generator().manual_seed(2100 + T)
    weight = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()
    wide_bank.set_pre_norm(weight, 1e-6)
    xbits = synthetic_np.tokens_bf16(T, H, 2200 + T)
    rbits = synthetic_np.tokens_bf16(T, H, 2300 + T)
    x, r = bits_to_bf16_tensor(xbits), bits_to_bf16_tensor(rbits)
    want = wide_bank.forward(x, residual=r, pre_norm=True)
    torch.cuda.synchronize()
    want = want.cpu().view(torch.int16).numpy()
    hx = torch.from_numpy(xbits.view(np.int16)).view(torch.bfloat16).pin_memory()
    hr = torch.from_numpy(rbits.view(np.int16)).view(torch.bfloat16).pin_memory()
    for out in (torch.empty(T, H, dtype=torch.bfloat16).pin_memory(), torch.empty(T, H, dtype=torch.bfloat16)):
        wide_bank.forward_host(hx, residual=hr, out=out, pre_norm=True)
        np.testing.assert_array_equal(out.view(torch.int16).numpy(), want)


def test_forward_more_than_64_tokens(cuda_runtime, small_bank, small_host):
    import torch

    T, H = 150, small_host.hidden
    xbits = synthetic_np.tokens_bf16(T, H, 51)
    rbits = synthetic_np.tokens_bf16(T, H, 52)
    out = small_bank.forward(bits_to_bf16_tensor(xbits), residual=bits_to_bf16_tensor(rbits))
    torch.cuda.synchronize()
    ref = moe_layer(small_host, synthetic_np.bf16_bits_to_f32(xbits), synthetic_np.bf16_bits_to_f32(rbits))
    got = bf16_tensor_to_f32(out)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL


def test_skewed_routing(cuda_runtime):
    import torch

    host = synthetic_np.make_bank(64, 256, 128, 61, skew=True)
    bank = upload_bank(cuda_runtime, host)
    T, H = 48, 256
    xbits = synthetic_np.tokens_bf16(T, H, 62)
    out = bank.forward(bits_to_bf16_tensor(xbits))
    torch.cuda.synchronize()
    ref = moe_layer(host, synthetic_np.bf16_bits_to_f32(xbits))
    check_routing(bank, ref, T)
    # Skew concentrates load on the top-ranked experts.
    assert ref.counts.max() >= 3 * ref.counts.mean()
    assert rel_rmse(bf16_tensor_to_f32(out), ref.out) <= REL_RMSE_TOL
    bank.close()


def test_config0_full_size_bank(cuda_runtime):
    """BASELINE config 0 and 1 shapes (256 x 512 experts, hidden 2048) with a
    GPU-generated bank; the oracle receives the selected experts' bytes."""
    import torch

    from vllm_nvfp4_cuda import synthetic

    E, H, I, seed = 256, 2048, 512, 0
    bank, meta = synthetic.build_bank(cuda_runtime, E, H, I, seed)
    for T in (1, 4, 32):
        x = synthetic.synthetic_tokens(T, H, seed + T)
        out = bank.forward(x)
        torch.cuda.synchronize()
        r = bank.last_routing(T)
        needed = sorted(set(r.ids.reshape(-1).tolist()))
        host = BankHost(E, H, I, meta.router_bf16.numpy().view(np.uint16), meta.shared_gate_bf16.numpy().view(np.uint16))
        for e in needed:
            for p in range(3):
                packed, scales, div = synthetic.synthetic_expert_projection(e, p, H, I, seed)
                host.projections[p][e] = QuantizedMatrix(packed.cpu().numpy(), scales.cpu().numpy(), div)
        xf = x.to(torch.float32).cpu().numpy()
        ref = moe_layer(host, xf)
        check_routing(bank, ref, T)
        got = bf16_tensor_to_f32(out)
        assert rel_rmse(got, ref.out) <= REL_RMSE_TOL, T
        assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL, T
    bank.close()


def test_graph_primitives(cuda_runtime):
    rt = cuda_runtime
    rng = np.random.default_rng(5)
    n = 3000
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    ba, bb = rt.upload_buffer(a), rt.upload_buffer(b)
    out = rt.create_buffer(n * 4)
    rt.add_device(ba, bb, n, out)
    rt.synchronize()
    np.testing.assert_allclose(out.download((n,)), a + b, rtol=3e-5, atol=3e-5)
    rt.silu_mul_device(ba, bb, n, out)
    rt.synchronize()
    np.testing.assert_allclose(out.download((n,)), a / (1 + np.exp(-a)) * b, rtol=3e-5, atol=3e-5)
    rt.weighted_accumulate_device(ba, 0.5, out, n, reset=True)
    rt.weighted_accumulate_device(bb, 2.0, out, n)
    rt.synchronize()
    np.testing.assert_allclose(out.download((n,)), 0.5 * a + 2.0 * b, rtol=3e-5, atol=3e-5)
    rows, cols = 3, 1000
    w = (rng.standard_normal(cols).astype(np.float32) + 1).astype(np.float32)
    bw = rt.upload_buffer(w)
    rt.rmsnorm_device(ba, bw, rows, cols, 1e-6, out)
    rt.synchronize()
    xa = a[: rows * cols].reshape(rows, cols)
    ref = xa / np.sqrt(np.mean(xa * xa, axis=1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(out.download((rows, cols)), ref, rtol=3e-5, atol=3e-5)
    # BF16 GEMV primitive (FP64 accumulation) against the exact dot product.
    wr = synthetic_np.router_bf16(40, 256, 9)
    x = rng.standard_normal(256).astype(np.float32)
    bw16, bx = rt.upload_buffer(np.ascontiguousarray(wr)), rt.upload_buffer(x)
    bo = rt.create_buffer(40 * 4)
    rt.bf16_gemv_device(bw16, bx, 40, 256, bo)
    rt.synchronize()
    exact = synthetic_np.bf16_bits_to_f32(wr).astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(bo.download((40,)), exact, rtol=1e-6, atol=1e-6)
    for buf in (ba, bb, out, bw, bw16, bx, bo):
        buf.close()


def test_trace_profile_and_errors(cuda_runtime, small_bank, small_host):
    rt = cuda_runtime
    H = small_host.hidden
    x = rt.upload_buffer(np.zeros(H, dtype=np.float32))
    out = rt.create_buffer(H * 4)
    # One token: routing, gate/up and down (the down kernel combines); with
    # the fused one-token kernel selected, that one kernel.
    for kernels, ops in (("tensor_core", ["moe_route", "moe_gate_up", "moe_down"]), ("fused_token", ["moe_token"])):
        small_bank.set_decode_kernels(kernels)
        rt.set_trace_enabled(True)
        rt.set_trace_scope("moe.layer.00.experts")
        small_bank.decode_device(x, out)
        prof = rt.synchronize()
        events = rt.trace_events()
        rt.set_trace_enabled(False)
        small_bank.set_decode_kernels("tensor_core")
        assert prof.kernel_ns > 0
        assert [e.operation for e in events] == ops
        assert events[0].scope == "moe.layer.00.experts" and events[0].duration_ns > 0
    # Argument validation mirrors the lab's messages and status codes.
    with pytest.raises(RuntimeError, match=r"\(1\): invalid MoE bank decode buffers"):
        small_bank.decode_device(x, rt.create_buffer(4))
    with pytest.raises(ValueError):
        small_bank.upload_projection(0, 3, np.zeros((1, 1), np.uint8), np.zeros((1, 1), np.uint8), 1.0)
    partial = rt.create_moe_bank(small_host.router_bf16, small_host.shared_gate_bf16, small_host.intermediate)
    with pytest.raises(RuntimeError, match="requires every routed and shared projection"):
        partial.decode_device(x, out)
    partial.close()
    x.close()
    out.close()
