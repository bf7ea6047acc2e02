"""The allocation-free routing entry point (nvfp4_moe_route_static_scratch).

It exists for callers that may not allocate device memory while they route
tokens -- their device memory is planned by the host framework, or
allocation is off limits on their latency path -- so its working memory is a
fixed array inside the library instead of cudaMalloc'd scratch. This test
calls it through the C ABI twice in a row (the array keeps the first call's
contents, so the second call checks that nothing stale leaks through) and
compares routing ids, weights, counts and the dispatch permutation with the
bank's own routing from the regular entry point. The file sorts last so a
run that stops at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import cpu_oracle, synthetic_np
from oracle.nvfp4_oracle import dispatch

from helpers import bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu


def test_static_scratch_routing_matches_bank(cuda_runtime):
    import torch

    rt = cuda_runtime
    E, H, I = 64, 512, 128
    host = synthetic_np.make_bank(E, H, I, 77)
    bank = upload_bank(rt, host)
    router = bits_to_bf16_tensor(np.ascontiguousarray(host.router_all()))
    try:
        for call, T in enumerate((37, 64)):
            xbits = synthetic_np.tokens_bf16(T, H, 300 + call)
            x = bits_to_bf16_tensor(xbits)
            bank.forward(x)
            torch.cuda.synchronize()
            expected = bank.last_routing(T)

            ids = torch.full((T, 9), -1, dtype=torch.int32, device="cuda")
            weights = torch.zeros((T, 9), dtype=torch.float32, device="cuda")
            counts = torch.full((E,), -1, dtype=torch.int32, device="cuda")
            perm = torch.full((T * 8,), -1, dtype=torch.int32, device="cuda")
            stream = torch.cuda.current_stream()
            status = rt.lib.nvfp4_moe_route_static_scratch(
                C.c_void_p(router.data_ptr()), C.c_void_p(x.data_ptr()), T, E, H,
                C.c_void_p(ids.data_ptr()), C.c_void_p(weights.data_ptr()), C.c_void_p(counts.data_ptr()),
                C.c_void_p(perm.data_ptr()), C.c_void_p(stream.cuda_stream))
            assert status == 0, rt.lib.nvfp4_last_error()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(ids.cpu().numpy(), expected.ids)
            np.testing.assert_allclose(weights.cpu().numpy(), expected.weights, rtol=2e-6, atol=1e-7)
            np.testing.assert_array_equal(counts.cpu().numpy(), expected.counts)
            np.testing.assert_array_equal(perm.cpu().numpy(), expected.perm)
        # Sizes beyond the fixed array's limits are rejected with a message.
        status = rt.lib.nvfp4_moe_route_static_scratch(
            C.c_void_p(router.data_ptr()), C.c_void_p(x.data_ptr()), 65, E, H,
            C.c_void_p(ids.data_ptr()), C.c_void_p(weights.data_ptr()), None, None, None)
        assert status == 1 and b"1 to 64 tokens" in rt.lib.nvfp4_last_error()
    finally:
        bank.close()


def test_static_scratch_routing_at_its_limits(cuda_runtime):
    """The largest accepted call (256 experts, hidden 4096, 64 tokens: the
    carve nearest the array's 1 MiB) against the CPU restatement of the
    routing, twice in a row; then sizes just past each limit are rejected."""
    import torch

    rt = cuda_runtime
    E, H, T = 256, 4096, 64
    router_all = np.concatenate([synthetic_np.router_bf16(E, H, 81), synthetic_np.shared_gate_bf16(H, 81)[None]])
    router = bits_to_bf16_tensor(np.ascontiguousarray(router_all))
    stream = torch.cuda.current_stream()
    for call in range(2):
        xbits = synthetic_np.tokens_bf16(T, H, 900 + call)
        x = bits_to_bf16_tensor(xbits)
        ids = torch.full((T, 9), -1, dtype=torch.int32, device="cuda")
        weights = torch.zeros((T, 9), dtype=torch.float32, device="cuda")
        counts = torch.full((E,), -1, dtype=torch.int32, device="cuda")
        perm = torch.full((T * 8,), -1, dtype=torch.int32, device="cuda")
        status = rt.lib.nvfp4_moe_route_static_scratch(
            C.c_void_p(router.data_ptr()), C.c_void_p(x.data_ptr()), T, E, H,
            C.c_void_p(ids.data_ptr()), C.c_void_p(weights.data_ptr()), C.c_void_p(counts.data_ptr()),
            C.c_void_p(perm.data_ptr()), C.c_void_p(stream.cuda_stream))
        assert status == 0, rt.lib.nvfp4_last_error()
        torch.cuda.synchronize()
        ref_ids, ref_w, _ = cpu_oracle.route(router_all, synthetic_np.bf16_bits_to_f32(xbits))
        ref_counts, _, ref_perm = dispatch(ref_ids[:, :8], E)
        np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
        np.testing.assert_allclose(weights.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)
        np.testing.assert_array_equal(counts.cpu().numpy(), ref_counts)
        np.testing.assert_array_equal(perm.cpu().numpy(), ref_perm)
    for tokens, experts, hidden, msg in ((T, E, 4224, b"at most 4096"), (T, 257, 2048, b"8 to 256 experts"),
                                         (T, 7, 2048, b"8 to 256 experts"), (T, E, 2000, b"multiple of 128")):
        status = rt.lib.nvfp4_moe_route_static_scratch(
            C.c_void_p(router.data_ptr()), C.c_void_p(x.data_ptr()), tokens, experts, hidden,
            C.c_void_p(ids.data_ptr()), C.c_void_p(weights.data_ptr()), None, None, None)
        assert status == 1 and msg in rt.lib.nvfp4_last_error(), (tokens, experts, hidden)
