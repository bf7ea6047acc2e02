"""The one-token kernel (moe_token_kernel: the whole layer call in one
persistent grid) against the oracle, through the C ABI (needs an sm_100a
GPU).

One-token calls of a bank computing every expert run this kernel when the
bank's decode kernels are "fused_token" (opt-in). For each shape it serves (H a multiple of 256 up to 2048, I a multiple of
128 up to 1024):

* router logits equal the oracle's bit for bit (same FP32 order), ids,
  weights, counts and the dispatch permutation exactly;
* the output meets the BASELINE bound against the FP32 oracle with and
  without the residual, over consecutive calls (the grid barriers' words
  must come back to rest after every call) with different tokens;
* it agrees with the three-launch in-register path on the same token within
  the same bound;
* the lab's FP32 entry point (nvfp4_moe_bank_decode_device_enqueue_f32) and
  a skewed router bias take the same kernel;
* captured in a CUDA graph (a cooperative kernel node), replays give the
  eager call's bits.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import BankHost, QuantizedMatrix, max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

SHAPES = [(16, 256, 128, False), (64, 1024, 256, True), (32, 512, 1024, False), (256, 512, 512, True)]


def _check(bank, host, T, seed, residual):
    import torch

    xbits = synthetic_np.tokens_bf16(T, host.hidden, seed)
    rbits = synthetic_np.tokens_bf16(T, host.hidden, seed + 1) if residual else None
    out = bank.forward(bits_to_bf16_tensor(xbits), residual=bits_to_bf16_tensor(rbits) if residual else None)
    torch.cuda.synchronize()
    xf = synthetic_np.bf16_bits_to_f32(xbits)
    rf = synthetic_np.bf16_bits_to_f32(rbits) if residual else None
    ref = moe_layer(host, xf, rf)
    np.testing.assert_array_equal(bank.last_logits(T).view(np.uint32), ref.logits.view(np.uint32))
    r = bank.last_routing(T)
    np.testing.assert_array_equal(r.ids, ref.ids)
    np.testing.assert_allclose(r.weights, ref.weights, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(r.counts, ref.counts)
    np.testing.assert_array_equal(r.perm, ref.perm)
    got = bf16_tensor_to_f32(out)
    assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    return got, ref


@pytest.mark.parametrize("E,H,I,skew", SHAPES)
def test_token_kernel_shapes(cuda_runtime, E, H, I, skew):
    host = synthetic_np.make_bank(E, H, I, 400 + E + H + I, skew=skew)
    bank = upload_bank(cuda_runtime, host)
    bank.set_decode_kernels("fused_token")
    try:
        for call in range(3):
            _check(bank, host, 1, 50 + call, residual=call != 1)
        # The in-register path on the same token.
        got, ref = _check(bank, host, 1, 60, residual=False)
        bank.set_decode_kernels("in_register")
        try:
            other, _ = _check(bank, host, 1, 60, residual=False)
        finally:
            bank.set_decode_kernels("fused_token")
        assert rel_rmse(got, other) <= 2 * REL_RMSE_TOL
    finally:
        bank.close()


def test_token_kernel_reference_f32_abi(cuda_runtime):
    host = synthetic_np.make_bank(64, 1024, 256, 77)
    bank = upload_bank(cuda_runtime, host)
    bank.set_decode_kernels("fused_token")
    rt = cuda_runtime
    try:
        for seed in (3, 4):
            x = (synthetic_np.tokens_f32(1, host.hidden, seed) * np.float32(0.2)).astype(np.float32)
            xb = rt.upload_buffer(np.ascontiguousarray(x[0]))
            out = rt.create_buffer(host.hidden * 4)
            bank.decode_device(xb, out)
            rt.synchronize()
            got = out.download((1, host.hidden))
            ref = moe_layer(host, x)
            np.testing.assert_array_equal(bank.last_logits(1).view(np.uint32), ref.logits.view(np.uint32))
            np.testing.assert_array_equal(bank.last_routing(1).ids, ref.ids)
            assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
            assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
            xb.close()
            out.close()
    finally:
        bank.close()


def test_token_kernel_full_size_many_calls(cuda_runtime):
    """BASELINE config 0 (256 x 512 experts, hidden 2048) on a GPU-generated
    bank: 20 consecutive one-token calls, every fifth checked against the
    oracle on the experts it selected."""
    import torch

    from vllm_nvfp4_cuda import synthetic

    E, H, I, seed = 256, 2048, 512, 3
    bank, meta = synthetic.build_bank(cuda_runtime, E, H, I, seed)
    bank.set_decode_kernels("fused_token")
    host = BankHost(E, H, I, meta.router_bf16.numpy().view(np.uint16), meta.shared_gate_bf16.numpy().view(np.uint16))
    try:
        for call in range(20):
            x = synthetic.synthetic_tokens(1, H, 900 + call)
            r = synthetic.synthetic_tokens(1, H, 950 + call)
            out = bank.forward(x, residual=r)
            if call % 5:
                continue
            torch.cuda.synchronize()
            ids = bank.last_routing(1).ids
            for e in sorted(set(ids.reshape(-1).tolist())):
                if e not in host.projections[0]:
                    for p in range(3):
                        packed, scales, div = synthetic.synthetic_expert_projection(e, p, H, I, seed)
                        host.projections[p][e] = QuantizedMatrix(packed.cpu().numpy(), scales.cpu().numpy(), div)
            xf, rf = x.float().cpu().numpy(), r.float().cpu().numpy()
            ref = moe_layer(host, xf, rf)
            np.testing.assert_array_equal(ids, ref.ids)
            got = bf16_tensor_to_f32(out)
            assert rel_rmse(got, ref.out) <= REL_RMSE_TOL, call
            assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL, call
    finally:
        bank.close()


def test_token_kernel_in_cuda_graph(cuda_runtime):
    """The one-token kernel captured in a CUDA graph (a cooperative kernel
    node) replays to the eager call's bits, call after call."""
    import torch

    host = synthetic_np.make_bank(32, 512, 256, 88)
    bank = upload_bank(cuda_runtime, host)
    bank.set_decode_kernels("fused_token")
    try:
        xin = torch.empty(1, host.hidden, dtype=torch.bfloat16, device="cuda")
        res = bits_to_bf16_tensor(synthetic_np.tokens_bf16(1, host.hidden, 5))
        out = torch.empty_like(xin)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            bank.forward(xin, residual=res, out=out, stream=stream)  # eager warm-up outside the capture
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            bank.forward(xin, residual=res, out=out, stream=stream)
        for seed in (6, 7, 8):
            xbits = synthetic_np.tokens_bf16(1, host.hidden, seed)
            xin.copy_(bits_to_bf16_tensor(xbits))
            graph.replay()
            torch.cuda.synchronize()
            replayed = out.clone()
            eager = bank.forward(xin, residual=res)
            torch.cuda.synchronize()
            assert torch.equal(replayed, eager), seed
        del graph
    finally:
        bank.close()
