"""Expert-parallel kernels on one GPU (needs an sm_100a GPU).

Two banks with complementary expert ranges stand in for two ranks: each
computes its FP32 partial sum (NVFP4_MOE_PARTIAL_F32), the partials are added
(the collective's job across GPUs) and finalize_bf16 rounds the sum. The
result must match the single bank that computes every expert (only the order
of FP32 additions differs, then BF16 rounding), each partial must match the
oracle's partial layer, and routing must be identical on both banks. The
second bank receives only the projections of the experts it computes.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

E, H, I = 32, 512, 256


@pytest.fixture(scope="module")
def ep_host():
    return synthetic_np.make_bank(E, H, I, 71)


@pytest.fixture(scope="module")
def ep_banks(cuda_runtime, ep_host):
    full = upload_bank(cuda_runtime, ep_host)
    a = upload_bank(cuda_runtime, ep_host)
    a.set_expert_range(0, E // 2, True)
    # Rank 1 holds only its own experts' projections.
    h = ep_host
    b = cuda_runtime.create_moe_bank(np.ascontiguousarray(h.router_bf16), np.ascontiguousarray(h.shared_gate_bf16),
                                     h.intermediate)
    b.set_expert_range(E // 2, E // 2, False)
    for e in range(E // 2, E):
        for p in range(3):
            q = h.projections[p][e]
            b.upload_projection(e, p, np.ascontiguousarray(q.packed), np.ascontiguousarray(q.scales),
                                q.global_scale)
    yield full, a, b
    for bank in (full, a, b):
        bank.close()


@pytest.mark.parametrize("T", [1, 16, 32, 48, 64, 200])
def test_two_ranges_add_up_to_the_layer(cuda_runtime, ep_host, ep_banks, T):
    import torch

    full, a, b = ep_banks
    xbits = synthetic_np.tokens_bf16(T, H, 800 + T)
    rbits = synthetic_np.tokens_bf16(T, H, 900 + T)
    x, r = bits_to_bf16_tensor(xbits), bits_to_bf16_tensor(rbits)
    ref_bank = full.forward(x, residual=r)
    pa = a.forward_partial(x, residual=r)
    pb = b.forward_partial(x)
    out = cuda_runtime.finalize_bf16(pa + pb)
    torch.cuda.synchronize()
    for bank in (a, b):
        got_r, ref_r = bank.last_routing(T), full.last_routing(T)
        np.testing.assert_array_equal(got_r.ids, ref_r.ids)
        np.testing.assert_array_equal(got_r.perm, ref_r.perm)
    got = bf16_tensor_to_f32(out)
    assert rel_rmse(got, bf16_tensor_to_f32(ref_bank)) <= 1e-3
    xf, rf = synthetic_np.bf16_bits_to_f32(xbits), synthetic_np.bf16_bits_to_f32(rbits)
    fp32 = moe_layer(ep_host, xf, rf)
    assert rel_rmse(got, fp32.out) <= REL_RMSE_TOL
    assert max_abs_rel(got, fp32.out) <= MAX_ABS_REL_TOL
    part_b = moe_layer(ep_host, xf, None, expert_range=(E // 2, E // 2), shared_here=False).out
    assert rel_rmse(pb.cpu().numpy(), part_b) <= REL_RMSE_TOL


def test_finalize_adds_residual(cuda_runtime):
    import torch

    s = torch.randn(3, 64, device="cuda", dtype=torch.float32)
    r = torch.randn(3, 64, device="cuda").to(torch.bfloat16)
    out = cuda_runtime.finalize_bf16(s, residual=r)
    torch.cuda.synchronize()
    ref = (s + r.float()).to(torch.bfloat16)
    assert torch.equal(out, ref)


def test_forward_needs_owned_projections_only(cuda_runtime, ep_host, ep_banks):
    _, _, b = ep_banks
    b.set_expert_range(0, E, True)   # now claims experts it never received
    try:
        with pytest.raises(RuntimeError):
            b.forward_partial(bits_to_bf16_tensor(synthetic_np.tokens_bf16(2, H, 5)))
    finally:
        b.set_expert_range(E // 2, E // 2, False)


def test_fused_combine_single_rank_matches_forward(cuda_runtime, ep_host, ep_banks):
    """A one-rank context runs the fused combine without peers: the output must
    equal the plain forward bit for bit (same additions in the same order),
    over several calls (both buffer parities) and both decode variants."""
    import torch

    from vllm_nvfp4_cuda.runtime import EpContext

    full, _, _ = ep_banks
    ep = EpContext(cuda_runtime, 0, 1, 64, H)
    ep.open_peers([ep.ipc_handle()])
    try:
        for T in (1, 16, 32, 64, 16):
            x = bits_to_bf16_tensor(synthetic_np.tokens_bf16(T, H, 1200 + T))
            r = bits_to_bf16_tensor(synthetic_np.tokens_bf16(T, H, 1300 + T))
            ref = full.forward(x, residual=r)
            got = full.forward_ep(ep, x, residual=r)
            torch.cuda.synchronize()
            cuda_runtime.synchronize()
            assert torch.equal(got, ref), T
        with pytest.raises(RuntimeError):
            full.forward_ep(ep, bits_to_bf16_tensor(synthetic_np.tokens_bf16(65, H, 1)))
    finally:
        ep.close()
