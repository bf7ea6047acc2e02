"""Failure detection of the fused expert-parallel combine (needs an sm_100a GPU).

Rank 0 of a two-rank context runs a layer call whose peer never makes the
call: the peer is a child process that maps its buffers, hands over its
CUDA IPC handle and then only waits, launching nothing. The combine kernel's
wait for the peer's partial tiles is bounded by wall-clock time (1 s); it
must give up, record wait site 41 in the context's error word, and return,
so that ``synchronize`` raises INTERNAL (status 4) naming the site and the
runtime stays usable: a plain forward afterwards still matches the oracle.
The failure is made on the host (a rank that never joins), not on the GPU:
no kernel faults or spins without a bound, and nothing else waits on the
timed-out kernel.
"""

from __future__ import annotations

import time

import numpy as np
import pytest

from oracle import synthetic_np
from oracle.nvfp4_oracle import max_abs_rel, moe_layer, rel_rmse

from helpers import MAX_ABS_REL_TOL, REL_RMSE_TOL, bf16_tensor_to_f32, bits_to_bf16_tensor, upload_bank

pytestmark = pytest.mark.gpu

E, H, I = 32, 512, 256


def _silent_peer(conn, hidden):
    """Rank 1: map the context's buffers, send the IPC handle, then wait for
    the parent to finish -- never running a layer call."""
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (root, root / "x2-nvfp4-lab_b200"):
        sys.path.insert(0, str(p))
    from vllm_nvfp4_cuda.runtime import EpContext, Runtime

    rt = Runtime()
    ep = EpContext(rt, 1, 2, 64, hidden)
    conn.send(ep.ipc_handle())
    conn.recv()
    ep.close()
    rt.close()


def test_fused_combine_times_out_when_peer_never_calls(cuda_runtime):
    import multiprocessing as mp

    import torch

    from vllm_nvfp4_cuda.runtime import EpContext

    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_silent_peer, args=(child, H), daemon=True)
    proc.start()
    ep = None
    host = synthetic_np.make_bank(E, H, I, 31)
    bank = upload_bank(cuda_runtime, host)
    try:
        assert parent.poll(120), "peer process did not start"
        peer_handle = parent.recv()
        ep = EpContext(cuda_runtime, 0, 2, 64, H)
        ep.open_peers([ep.ipc_handle(), peer_handle])
        bank.set_expert_range(0, E // 2, True)
        x = bits_to_bf16_tensor(synthetic_np.tokens_bf16(4, H, 77))
        t0 = time.perf_counter()
        bank.forward_ep(ep, x)
        # The call runs on torch's stream: drain it, then the runtime's
        # synchronize reports what its kernels recorded.
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match=r"\(4\).*wait site 41"):
            cuda_runtime.synchronize()
        elapsed = time.perf_counter() - t0
        assert 0.5 < elapsed < 30.0, elapsed
        # The runtime and the bank remain usable after the timeout.
        bank.set_expert_range(0, E, True)
        xbits = synthetic_np.tokens_bf16(3, H, 78)
        out = bank.forward(bits_to_bf16_tensor(xbits))
        torch.cuda.synchronize()
        cuda_runtime.synchronize()
        ref = moe_layer(host, synthetic_np.bf16_bits_to_f32(xbits))
        got = bf16_tensor_to_f32(out)
        assert rel_rmse(got, ref.out) <= REL_RMSE_TOL
        assert max_abs_rel(got, ref.out) <= MAX_ABS_REL_TOL
    finally:
        if ep is not None:
            ep.close()
        bank.close()
        parent.send("done")
        proc.join(60)
    assert proc.exitcode == 0
