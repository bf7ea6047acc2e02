"""Benchmark of the NVFP4 MoE layer on B200 (driver contract: one JSON line).

Workload (the decode metric's batched configuration):
one Qwen3.5-MoE-shape layer (hidden 2048, 256 routed experts x intermediate
512, top-8 + shared expert), 32 independent BF16 tokens per step, all 257
experts resident in HBM. A step is one layer forward over one batch. Inputs
rotate through a pool of distinct token batches (so the routed experts
change step to step) and L2 is flushed before every step, outside that
step's CUDA-event pair: a 256 MiB write, then a 256 MiB read, so the
write's dirty lines reach HBM before the step instead of inside it (a
write-only flush adds ~126 MB of write-backs to the timed step, which a
layer's own few MB of writes never cause; the line also reports the step
under the write-only flush, `ms_per_step_write_only_flush`).

  value      tokens/s over all ranks, device time (sum of per-step events,
             max over ranks)
  e2e        the same metric end to end with host buffers, wall clock:
             one nvfp4_moe_bank_forward_host_bf16 call per step (pinned
             host x and residual -> device, the forward, the output back to
             pinned host memory, one stream synchronize)
  roofline   dominant kernel (moe_gate_up): algorithmic bytes per launch /
             its average CUDA-event duration, against MEASURED_PEAKS hbm_gbs
  cpu_baseline  the C restatement of the lab's CPU path (oracle/cpu_moe.c)
             on this host's cores, on a bounded sample
  linear     the dense NVFP4 linear at the LM-head shape (248320 x 2048),
             1 and 4 vectors: device time per call and its HBM rate

--gpus N (under torchrun) runs the layer expert-parallel over the N GPUs:
rank r holds routed experts [r*256/N, (r+1)*256/N) and the shared expert on
rank 0, every rank sees the same 32 tokens (strong scaling: the step's work
is fixed), and the combine kernel reduces the ranks' partial tiles over
NVLink peer memory (no NCCL call on the step's path). `value` is the 32
tokens over the step time (max over ranks); `step_breakdown` splits the
step into routing, expert GEMVs and the exchange. The `expert_parallel`
object adds the one-token and 4096-token calls (NCCL all-reduce) and the
token-sharded 4096-token prefill (NCCL all-to-all).
--impl reference times the lab's CPU path (the C restatement) for the same
workload, W untimed batches and then exactly K timed ones, each a batch of
--tokens tokens on all host cores, and prints its own JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_ROOT = ROOT / "x2-nvfp4-lab_b200"
for _p in (ROOT, PKG_ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

E, H, I = 256, 2048, 512
PER_PROJ_BYTES = H * I // 2 + H * I // 16  # packed + scales of one projection
METRIC = "MoE layer decode tokens/s (µs/token = 1e6 / value)"
UNIT = "tokens/s"
WORKLOAD = "config1_decode_batch32"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-prefill", action="store_true", help="skip the prefill legs (configs 2 and 3)")
    p.add_argument("--no-stack", action="store_true", help="skip the 40-layer stack leg (config 4)")
    p.add_argument("--no-linear", action="store_true", help="skip the dense NVFP4 linear leg (LM-head shape)")
    p.add_argument("--decode-kernels", choices=["tensor_core", "in_register", "fused_token"], default="tensor_core",
                   help="decode expert GEMVs (the library's default is tensor_core)")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


class L2Flush:
    """Evicts the layer's data from L2 (126 MB) before a timed step: a
    256 MiB write, then a 256 MiB read of another buffer, so the write's
    dirty lines are written back here and L2 holds clean, unrelated lines
    when the step starts (the state a layer meets after other layers'
    weight reads). Runs on the current stream."""

    def __init__(self):
        import torch

        self.w = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
        self.r = torch.ones(64 * 1024 * 1024, dtype=torch.int32, device="cuda")

    def __call__(self, write_only: bool = False) -> None:
        import torch

        self.w.zero_()
        if not write_only:
            torch.amax(self.r)


class ClockSampler:
    """SM clock and throttle reasons of one GPU sampled every 20 ms through
    NVML (read-only queries) while the timed region runs (one sample at
    entry, so a short region still has one)."""

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, index: int, interval: float = 0.005):
        self.index = index
        self.interval = interval
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((float(mhz), int(reasons)))
            except Exception:
                pass
            self._stop.wait(self.interval)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        reasons = sorted({name for _, bits in self.samples for name, mask in self.REASONS.items() if bits & mask})
        mhz = [m for m, _ in self.samples]
        return {
            "sm_mhz": statistics.median(mhz) if mhz else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(mhz),
        }


# --------------------------------------------------------------- CPU leg


def cpu_baseline_measure(tokens: int, seed: int, min_seconds: float = 10.0, max_steps: int = 200,
                         steps: int | None = None, warmup: int = 1) -> dict:
    """Time the C restatement of the lab's CPU path (oracle/cpu_moe.c) on a
    full-size synthetic bank: after `warmup` untimed batches, either exactly
    `steps` batches of `tokens` tokens or, when `steps` is None, batches until
    at least `min_seconds` of CPU work (at least 2, at most `max_steps`)."""
    import numpy as np

    from oracle import cpu_oracle, synthetic_np

    from vllm_nvfp4_cuda import synthetic

    threads = os.cpu_count() or 1
    # Full 257-expert bank generated on the host (torch CPU), device layout.
    meta = synthetic.synthetic_router(E, H, seed)
    packed = [np.empty((E + 1) * H * I // 2, dtype=np.uint8) for _ in range(3)]
    scales = [np.empty((E + 1) * H * I // 16, dtype=np.uint8) for _ in range(3)]
    inv = np.zeros((3, E + 1), dtype=np.float32)
    pp, ps = H * I // 2, H * I // 16
    for e in range(E + 1):
        for p in range(3):
            pk, sc, div = synthetic.synthetic_expert_projection(e, p, H, I, seed, device="cpu")
            packed[p][e * pp:(e + 1) * pp] = pk.numpy().reshape(-1)
            scales[p][e * ps:(e + 1) * ps] = sc.numpy().reshape(-1)
            inv[p, e] = np.float32(1.0) / np.float32(div)
    router = np.ascontiguousarray(np.concatenate(
        [meta.router_bf16.numpy().view(np.uint16), meta.shared_gate_bf16.numpy().view(np.uint16)[None]]))
    dense = cpu_oracle.DenseBank(E, H, I, packed, scales, inv, router, None)
    warm = synthetic_np.tokens_f32(tokens, H, seed + 998)
    for _ in range(max(1, warmup)):
        dense.forward(warm, threads=threads)
    xs = [synthetic_np.tokens_f32(tokens, H, seed + s) for s in range(8)]
    done = 0
    t0 = time.perf_counter()
    while (done < steps) if steps is not None else (
            done < max_steps and (done < 2 or time.perf_counter() - t0 < min_seconds)):
        dense.forward(xs[done % len(xs)], threads=threads)
        done += 1
    dt = time.perf_counter() - t0
    steps = done
    return {
        "value": round(tokens * steps / dt, 3),
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{steps} steps x {tokens} tokens of {WORKLOAD} on the full 257-expert bank "
                  f"(C restatement of nvfp4_cpu.cpp neon_row + layer, {threads} threads)",
        "seconds": round(dt, 3),
    }


def run_reference(args) -> int:
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    steps, warmup = max(1, args.steps), max(1, args.warmup)
    cpu = cpu_baseline_measure(args.tokens, args.seed, steps=steps, warmup=warmup)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": cpu["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(1000.0 * args.tokens / cpu["value"], 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded BASELINE distributions; no checkpoint on this machine)",
        "config": {"workload": WORKLOAD, "tokens_per_step": args.tokens, "experts": E, "hidden": H,
                   "intermediate": I, "implementation": "lab CPU path restated in C (oracle/cpu_moe.c); "
                   "the NEON original needs arm_neon.h and does not build on x86-64"},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- GPU leg


def prefill_leg(rt, bank, stream, flush, T: int, seed: int, steps: int, warmup: int, skew: bool) -> dict:
    """BASELINE config 2 (T=4096) / config 3 (T=8192, skewed router) on the
    resident bank: device time per layer pass (L2 flushed before each pass,
    outside its events), per-kernel times from the runtime trace, tensor and
    HBM rates against the algorithmic work of one pass."""
    import numpy as np
    import torch

    from vllm_nvfp4_cuda import synthetic

    bias = synthetic.synthetic_router(E, H, seed, skew=True).router_bias.numpy() if skew else None
    bank.set_router_bias(bias)
    bank.reserve_prefill(T)
    pool = [synthetic.synthetic_tokens(T, H, 7000 + 17 * T + i) for i in range(2)]
    res = synthetic.synthetic_tokens(T, H, 9000 + T)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(warmup):
            flush()
            bank.forward(pool[i % 2], residual=res, out=out, stream=stream)
    stream.synchronize()
    r = bank.last_routing(T)
    counts = np.asarray(r.counts)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(2e6))
        for i in range(steps):
            flush()
            starts[i].record(stream)
            bank.forward(pool[i % 2], residual=res, out=out, stream=stream)
            ends[i].record(stream)
    stream.synchronize()
    rt.synchronize()
    by_op: dict[str, float] = {}
    traced = traced_steps(rt, stream, flush,
                          lambda i: bank.forward(pool[i % 2], residual=res, out=out, stream=stream), steps)
    for ev in traced:
        by_op[ev.operation] = by_op.get(ev.operation, 0.0) + ev.duration_ns / 1e3 / steps
    # Cross-check on a seeded sample of 32 tokens: the same rows through the
    # decode path (tensor-core GEMVs, four activation terms; itself tested
    # against the FP32 oracle), compared with this pass's output rows. The
    # hottest expert's tokens are in the sample when the load is skewed.
    g = torch.Generator().manual_seed(seed + T)
    r_ids = torch.as_tensor(r.ids[:, :8])
    hot = int(np.argmax(counts))
    hot_tokens = torch.nonzero((r_ids == hot).any(dim=1)).flatten()[:8]
    rest = torch.randperm(T, generator=g)[:32]
    sample = torch.unique(torch.cat([hot_tokens, rest]))[:32].to("cuda")
    with torch.cuda.stream(stream):
        bank.forward(pool[(steps - 1) % 2], residual=res, out=out, stream=stream)
        ref = bank.forward(pool[(steps - 1) % 2][sample].contiguous(), residual=res[sample].contiguous(),
                           stream=stream)
    stream.synchronize()
    rt.synchronize()
    got = out[sample].float()
    want = ref.float()
    diff = (got - want).norm() / want.norm()
    mar = ((got - want).abs().max() / want.abs().max()).item()
    parity = {"vs": "decode path (tensor-core GEMVs, four activation terms) on the same tokens",
              "tokens": int(sample.numel()), "hot_expert_tokens": int(hot_tokens.numel()),
              "rel_rmse": float(f"{diff.item():.3e}"), "max_abs_rel": float(f"{mar:.3e}")}
    if skew:
        bank.set_router_bias(None)
    ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    ms_pass = statistics.median(ms)
    flops = 9.0 * 6.0 * H * I * T                     # algorithmic: 9 slots x (gate, up, down) x 2 flop/MAC
    active = int((counts > 0).sum()) + 1
    hbm = active * 3 * PER_PROJ_BYTES + (E + 1) * H * 2 + 3 * T * H * 2
    gemm_us = by_op.get("moe_gate_up", 0.0) + by_op.get("moe_down", 0.0)
    return {
        "workload": "config3_prefill8192_skewed" if skew else "config2_prefill4096",
        "tokens": T,
        "tokens_per_s": round(T / (ms_pass / 1000.0), 1),
        "ms_per_pass": round(ms_pass, 4),
        "passes": steps,
        "kernels_us": {k: round(v, 2) for k, v in by_op.items()},
        "algorithmic_tflops": round(flops / (ms_pass / 1000.0) / 1e12, 1),
        "gemm_tflops": round(flops / (gemm_us / 1e6) / 1e12, 1) if gemm_us else None,
        "fp4_dense_nominal_tflops": 9000.0,
        "layer_hbm_gbs": round(hbm / (ms_pass / 1000.0) / 1e9, 1),
        "activation_terms": [4, 3],
        "max_expert_load": int(counts.max()),
        "mean_expert_load": round(float(counts.mean()), 1),
        "parity": parity,
    }


def stack_leg(rt, seed: int, steps: int, warmup: int, layers: int = 40, decode_kernels: str = "tensor_core") -> dict:
    """the resident decode stack of ``layers`` independently
    seeded layers (h <- h + MoE(RMSNorm(h)), attention omitted, the RMSNorm
    fused into each layer's forward), all banks in HBM, one CUDA graph per
    batch size replayed per step. Device time per
    step (CUDA events around each replay; the step's input is copied in
    before the start event); the weights a step streams (hundreds of MB)
    are far larger than L2, so no flush is needed. Algorithmic bytes per
    step: for every layer its routed experts' and the shared expert's three
    projections, the router and shared gate, and the hidden state in and out."""
    import numpy as np
    import torch

    from vllm_nvfp4_cuda import synthetic
    from vllm_nvfp4_cuda.stack import MoeStack

    banks = [synthetic.build_bank(rt, E, H, I, seed, layer=101 + layer)[0] for layer in range(layers)]
    for b in banks:
        b.set_decode_kernels(decode_kernels)
    stack = MoeStack(rt, banks)
    stream = torch.cuda.Stream()
    peak = measured_peaks().get("hbm_gbs")
    out = {"workload": "config4_stack40", "layers": layers, "l2": "not flushed (weights per step >> L2)",
           "launches_per_layer": "the layer call's decode kernels with the RMSNorm fused into routing up to 32 "
                                 "tokens (one RMSNorm launch more above); one CUDA graph per step"}
    for T in (1, 64):
        g = stack.capture(T)
        xs = [synthetic.synthetic_tokens(T, H, 12000 + 97 * T + i) for i in range(4)]
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        with torch.cuda.stream(stream):
            for i in range(warmup):
                g.run(xs[i % 4])
            for i in range(steps):
                g.input.copy_(xs[i % 4])
                starts[i].record(stream)
                g.replay()
                ends[i].record(stream)
        stream.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in zip(starts, ends))
        step_bytes = 0
        for b in banks:
            r = b.last_routing(T)
            uniq = len(set(np.asarray(r.ids)[:, :8].reshape(-1).tolist()))
            step_bytes += (uniq + 1) * 3 * PER_PROJ_BYTES + (E + 1) * H * 2 + 2 * T * H * 2
        gbs = step_bytes / (ms / 1000.0) / 1e9
        out[f"batch{T}"] = {
            "tokens_per_s": round(T / (ms / 1000.0), 1),
            "us_per_step": round(ms * 1000.0, 2),
            "us_per_layer": round(ms * 1000.0 / layers, 2),
            "algorithmic_mb_per_step": round(step_bytes / 1e6, 1),
            "hbm_gbs": round(gbs, 1),
            "hbm_frac_of_measured": round(gbs / peak, 4) if peak else None,
        }
        g.close()
        del g
    for b in banks:
        b.close()
    return out


def linear_leg(rt, seed: int, steps: int, warmup: int, rows: int = 248320, cols: int = 2048) -> dict:
    """The dense NVFP4 linear (the lab's nvfp4_linear entry points behind its
    vLLM provider) at the LM-head shape, 248320 x 2048, for 1 and 4 FP32
    vectors through the tensor entry point on a torch stream: the activations'
    NVFP4 terms, then the tensor-core weight stream (two launches). Device
    time per call (CUDA events, median); the 286 MB of weights a call streams
    are far larger than L2, so no flush is needed. Algorithmic bytes per call:
    packed codes and scales (0.5625 B per weight) plus x in and y out in FP32."""
    import numpy as np
    import torch

    rng = np.random.default_rng(seed + 77)
    packed = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(0x30, 0x48, size=(rows, cols // 16), dtype=np.uint8)
    m = rt.upload(packed, scales, 1.0)
    del packed, scales
    stream = torch.cuda.Stream()
    peak = measured_peaks().get("hbm_gbs")
    out = {"workload": f"lm_head_{rows}x{cols}", "l2": "not flushed (weights per call >> L2)",
           "kernel": "linear_terms_kernel + linear_tc_kernel (tcgen05 kind::mxf4nvf4)", "launches_per_call": 2}
    try:
        for V in (1, 4):
            x = torch.from_numpy(rng.standard_normal((V, cols)).astype(np.float32)).cuda()
            y = torch.empty(V, rows, dtype=torch.float32, device="cuda")
            stream.wait_stream(torch.cuda.current_stream())
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            with torch.cuda.stream(stream):
                for _ in range(warmup):
                    rt.linear_tensor(m, x, out=y, stream=stream)
                for i in range(steps):
                    starts[i].record(stream)
                    rt.linear_tensor(m, x, out=y, stream=stream)
                    ends[i].record(stream)
            stream.synchronize()
            ms = statistics.median(a.elapsed_time(b) for a, b in zip(starts, ends))
            nbytes = rows * cols * 9 // 16 + V * (rows + cols) * 4
            gbs = nbytes / (ms / 1000.0) / 1e9
            out[f"vectors{V}"] = {
                "us_per_call": round(ms * 1000.0, 2),
                "algorithmic_mb": round(nbytes / 1e6, 1),
                "hbm_gbs": round(gbs, 1),
                "hbm_frac_of_measured": round(gbs / peak, 4) if peak else None,
            }
    finally:
        m.close()
    return out


def ep_leg(rt, bank, stream, flush, pg, world: int, seed: int, steps: int, warmup: int) -> dict:
    """Expert parallelism across the job's GPUs: rank r holds routed experts
    [r*E/N, (r+1)*E/N) (the shared expert on rank 0), the tokens are the same
    on every rank. Two reductions of the ranks' partial sums: NCCL all-reduce
    of FP32 partials + finalize (every size), and the combine fused with the
    reduction over NVLink peer memory (calls of up to 64 tokens). Per-call
    device time (CUDA events on the launching stream, L2 flushed before each
    call, max over ranks), and each output's relative RMSE against the
    single-GPU bank (full expert range) on the same tokens."""
    import torch

    from vllm_nvfp4_cuda import synthetic
    from vllm_nvfp4_cuda.expert_parallel import ExpertParallelLayer

    cases = (("decode_batch32", 32), ("decode_one_token", 1), ("prefill4096", 4096))
    data = {name: (synthetic.synthetic_tokens(T, H, seed + 70), synthetic.synthetic_tokens(T, H, seed + 71))
            for name, T in cases}
    refs = {name: bank.forward(x, residual=r).float() for name, (x, r) in data.items()}
    torch.cuda.synchronize()
    finalize = lambda t: rt.finalize_bf16(t)  # noqa: E731
    align_buf = torch.zeros(1, device="cuda")
    layers = {"nccl_all_reduce": ExpertParallelLayer(bank, finalize),
              "fused_combine_p2p": ExpertParallelLayer(bank, finalize, fused_runtime=rt)}
    out = {"ranks": world, "experts_per_rank": layers["nccl_all_reduce"].range.count,
           "reductions": {"nccl_all_reduce": "NCCL all_reduce of the FP32 [tokens, hidden] partials + finalize",
                          "fused_combine_p2p": "combine kernel reads every rank's partial tile over NVLink"},
           "calls": {}}
    for kind, layer in layers.items():
        for name, T in cases:
            if kind == "fused_combine_p2p" and T > 64:
                continue
            x, r = data[name]
            n = steps if T <= 64 else min(steps, 10)
            with torch.cuda.stream(stream):
                for _ in range(warmup):
                    flush()
                    y = layer.forward(x, r)
            stream.synchronize()
            err = float(((y.float() - refs[name]).pow(2).mean() / refs[name].pow(2).mean()).sqrt())
            pg.barrier()
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
            with torch.cuda.stream(stream):
                torch.cuda._sleep(int(2e5) * n)
                # Start every rank's first call together (both reductions
                # synchronise the ranks at every call after that).
                pg.all_reduce(align_buf)
                for i in range(n):
                    flush()
                    ev[i][0].record(stream)
                    layer.forward(x, r)
                    ev[i][1].record(stream)
            stream.synchronize()
            rt.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in ev) / n
            t = torch.tensor([ms, err], device="cuda", dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms, err = float(t[0].item()), float(t[1].item())
            out["calls"].setdefault(kind, {})[name] = {
                "tokens": T, "us_per_call": round(ms * 1000.0, 2), "tokens_per_s": round(T / (ms / 1000.0), 1),
                "rel_rmse_vs_single_gpu": float(f"{err:.3g}")}
    layers["fused_combine_p2p"].close()
    pg.barrier()
    bank.set_expert_range(0, E, True)
    out["token_sharded_prefill4096"] = token_sharded_leg(bank, rt, pg, world, seed)
    bank.set_expert_range(0, E, True)
    return out


def token_sharded_leg(bank, rt, pg, world: int, seed: int, T: int = 4096, calls: int = 5) -> dict:
    """BASELINE config 2 with the tokens sharded: rank r brings T/N tokens,
    routes them, ships each token row once to every other rank owning one
    of its picks (NCCL all-to-all), computes the rows it received over its
    own experts and returns the FP32 partials (TokenShardedLayer). The
    composition synchronises with the host (counts), so each call is timed
    by wall clock between barriers, max over ranks; outputs are compared
    with the single-GPU bank on the same tokens."""
    import torch

    from vllm_nvfp4_cuda import synthetic
    from vllm_nvfp4_cuda.expert_parallel import TokenShardedLayer

    rank = pg.get_rank()
    per = T // world
    x_all = synthetic.synthetic_tokens(T, H, seed + 80)
    r_all = synthetic.synthetic_tokens(T, H, seed + 81)
    ref = bank.forward(x_all, residual=r_all).float()[rank * per:(rank + 1) * per]
    x = x_all[rank * per:(rank + 1) * per].contiguous()
    r = r_all[rank * per:(rank + 1) * per].contiguous()
    torch.cuda.synchronize()
    layer = TokenShardedLayer(bank, lambda t: rt.finalize_bf16(t))
    y = layer.forward(x, r)
    torch.cuda.synchronize()
    err = float(((y.float() - ref).pow(2).mean() / ref.pow(2).mean()).sqrt())
    times = []
    for _ in range(calls):
        pg.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layer.forward(x, r)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    t = torch.tensor([min(times), err], device="cuda", dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    sec, err = float(t[0].item()), float(t[1].item())
    return {"tokens": T, "tokens_per_rank": per, "ms_per_call": round(sec * 1000.0, 3),
            "tokens_per_s": round(T / sec, 1), "rel_rmse_vs_single_gpu": float(f"{err:.3g}"),
            "timing": "wall clock per call between barriers (the composition syncs with the host), best of "
                      f"{calls}, max over ranks"}


def traced_steps(rt, stream, flush, step, n: int, align=None):
    """Run `step(i)` n times with the runtime trace on (L2 flushed before each
    step) and return the trace events: per-kernel device durations."""
    import torch

    torch.cuda.synchronize()
    rt.set_trace_enabled(True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(2e5) * n)
        if align is not None:
            align()
        for i in range(n):
            flush()
            step(i)
    stream.synchronize()
    rt.synchronize()
    events = rt.trace_events()
    rt.set_trace_enabled(False)
    return events


def run_ours(args) -> int:
    import numpy as np
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist

    from vllm_nvfp4_cuda import synthetic
    from vllm_nvfp4_cuda.runtime import Runtime

    T = args.tokens
    # The library runs calls of 4 to 32 tokens on the tensor-core expert
    # GEMVs for this shape (five launches per layer call), others in-register
    # (three launches up to 16 tokens, where the down kernel combines; four
    # above). Under expert parallelism the combine is the cross-rank one.
    tc_decode = 4 <= T <= 32 and args.decode_kernels == "tensor_core"
    launches = 5 if tc_decode else (3 if T <= 16 else 4)
    if world > 1:
        launches = 5 if tc_decode else 3
    rt = Runtime()
    bank, meta = synthetic.build_bank(rt, E, H, I, args.seed)
    bank.set_decode_kernels(args.decode_kernels)
    stream = torch.cuda.Stream()
    pool_n = 16
    # One GPU: the whole layer per rank. Several GPUs: expert parallelism --
    # rank r holds routed experts [r*E/N, (r+1)*E/N) (the shared expert on
    # rank 0), every rank sees the same 32 tokens, and the combine reduces
    # the ranks' partial tiles over NVLink peer memory in the same kernel.
    pool = [synthetic.synthetic_tokens(T, H, 1000 + i) for i in range(pool_n)]
    res_pool = [synthetic.synthetic_tokens(T, H, 5000 + i) for i in range(pool_n)]
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    flush = L2Flush()
    torch.cuda.synchronize()
    ep_layer = None
    first, count, shared_here = 0, E, True
    if world > 1:
        from vllm_nvfp4_cuda.expert_parallel import ExpertParallelLayer

        ep_layer = ExpertParallelLayer(bank, lambda t: rt.finalize_bf16(t), fused_runtime=rt)
        first, count, shared_here = ep_layer.range.first, ep_layer.range.count, ep_layer.range.shared_here

    def step(i):
        if ep_layer is not None:
            ep_layer.forward(pool[i % pool_n], residual=res_pool[i % pool_n], stream=stream)
        else:
            bank.forward(pool[i % pool_n], residual=res_pool[i % pool_n], out=out, stream=stream)

    # Routing of every pool batch -> algorithmic bytes of each step (this
    # rank's routed experts, plus the shared expert where it is computed).
    uniq = []
    for i in range(pool_n):
        with torch.cuda.stream(stream):
            step(i)
        stream.synchronize()
        r = bank.last_routing(T)
        ids = set(r.ids[:, :8].reshape(-1).tolist())
        uniq.append(len([e for e in ids if first <= e < first + count]) + (1 if shared_here else 0))
    gate_up_bytes = [u * 2 * PER_PROJ_BYTES + T * H * 2 + T * 9 * I * 2 for u in uniq]
    step_bytes = [u * 3 * PER_PROJ_BYTES + (E + 1) * H * 2 + 3 * T * H * 2 for u in uniq]

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            flush()
            step(i)
    stream.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()

    # Under expert parallelism every step ends in the cross-rank exchange, so
    # a rank's first timed step would also wait out the other ranks' host-side
    # launch skew; one all-reduce on the stream after the spin kernel starts
    # every rank's first step together (each step's exchange keeps them so).
    align_buf = torch.zeros(1, device="cuda") if pg else None

    def align():
        if pg:
            pg.all_reduce(align_buf)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # Clocks are sampled from the timed decode steps through the one-token and
    # prefill legs (all device-busy stretches).
    clocks = ClockSampler(local).__enter__()
    with torch.cuda.stream(stream):
        # A bounded spin kernel ahead of the first event lets the host
        # enqueue every step before the GPU reaches it, so each event
        # pair brackets device work only.
        torch.cuda._sleep(int(2e5) * args.steps)
        align()
        for i in range(args.steps):
            flush()
            starts[i].record(stream)
            step(i)
            ends[i].record(stream)
    stream.synchronize()
    rt.synchronize()
    # The same steps after a write-only flush, for comparison (reported, not
    # the headline).
    wo_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    wo_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(2e5) * args.steps)
        align()
        for i in range(args.steps):
            flush(write_only=True)
            wo_starts[i].record(stream)
            step(i)
            wo_ends[i].record(stream)
    stream.synchronize()
    rt.synchronize()
    # Per-kernel durations come from a second, traced pass over the same steps
    # (tracing records an event pair around every kernel, which would also
    # serialise the dependent launches of the timed pass).
    events = traced_steps(rt, stream, flush, step, args.steps, align if pg else None)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = float(sum(step_ms))
    wo_total_ms = float(sum(s.elapsed_time(e) for s, e in zip(wo_starts, wo_ends)))
    if pg:
        t = torch.tensor([total_ms, wo_total_ms], device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms, wo_total_ms = float(t[0].item()), float(t[1].item())
    value = T * args.steps / (total_ms / 1000.0)

    by_op: dict[str, list[float]] = {}
    for ev in events:
        by_op.setdefault(ev.operation, []).append(ev.duration_ns / 1e6)
    gu = by_op.get("moe_gate_up", [])
    gu_bytes = sum(gate_up_bytes[i % pool_n] for i in range(len(gu)))
    gu_ms = sum(gu)
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    achieved = gu_bytes / (gu_ms / 1000.0) / 1e9 if gu_ms > 0 else None
    traffic_path = ROOT / "profiles" / "traffic.json"
    traffic = None
    if traffic_path.exists() and world == 1:
        traffic = json.loads(traffic_path.read_text()).get(f"moe_gate_up_T{T}")
    layer_bytes = sum(step_bytes[i % pool_n] for i in range(args.steps))

    # Per-step breakdown (traced pass, this rank): routing, expert GEMVs,
    # and the cross-rank exchange (the fused combine) under expert parallelism.
    breakdown = {
        "routing_us": round(1000.0 * sum(by_op.get("moe_route", [])) / args.steps, 2),
        "experts_us": round(1000.0 * sum(sum(by_op.get(k, [])) for k in ("moe_gate_up", "moe_quantize_act",
                                                                      "moe_down")) / args.steps, 2),
        "exchange_us": round(1000.0 * sum(by_op.get("moe_combine_ep", [])) / args.steps, 2),
    }
    if ep_layer is not None:
        t = torch.tensor(list(breakdown.values()), device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        breakdown = dict(zip(breakdown, (round(float(v), 2) for v in t.tolist())))
        breakdown["note"] = "per-rank traced kernel times, max over ranks; traced kernels each include a launch gap"

    # T=1 latency (BASELINE config 0 target), same protocol, one GPU.
    lat = []
    t1_ops: dict[str, list[float]] = {}
    if world == 1:
        x1 = [p[:1].contiguous() for p in pool]
        o1 = torch.empty(1, H, dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(40)]
            torch.cuda._sleep(int(2e5) * 45)
            for i in range(45):
                flush()
                if i >= 5:
                    ev[i - 5][0].record(stream)
                bank.forward(x1[i % pool_n], out=o1, stream=stream)
                if i >= 5:
                    ev[i - 5][1].record(stream)
        stream.synchronize()
        rt.synchronize()
        lat = sorted(a.elapsed_time(b) * 1000.0 for a, b in ev)
        for evt in traced_steps(rt, stream, flush, lambda i: bank.forward(x1[i % pool_n], out=o1, stream=stream),
                                20):
            t1_ops.setdefault(evt.operation, []).append(evt.duration_ns / 1e3)

    # End to end: pinned host x and residual in, the layer, the output back
    # to pinned host memory, one synchronize per step.
    host_x = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(pool_n)]
    host_r = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(pool_n)]
    for i in range(pool_n):
        host_x[i].copy_(pool[i].cpu())
        host_r[i].copy_(res_pool[i].cpu())
    host_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    dev_x = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    dev_r = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def e2e_step(i):
        if ep_layer is None:
            # One call of the host entry point (nvfp4_moe_bank_forward_host_bf16).
            bank.forward_host(host_x[i % pool_n], residual=host_r[i % pool_n], out=host_out)
            return
        with torch.cuda.stream(stream):
            dev_x.copy_(host_x[i % pool_n], non_blocking=True)
            dev_r.copy_(host_r[i % pool_n], non_blocking=True)
            y = ep_layer.forward(dev_x, residual=dev_r, stream=stream)
            host_out.copy_(y, non_blocking=True)
        stream.synchronize()

    for i in range(args.warmup):
        e2e_step(i)
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e_s = time.perf_counter() - t0
    if pg:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = T * args.steps / e2e_s

    if ep_layer is not None:
        ep_layer.close()
        pg.barrier()
        bank.set_expert_range(0, E, True)

    ep = None
    if world > 1:
        ep = ep_leg(rt, bank, stream, flush, pg, world, args.seed, args.steps, 3)

    prefill = []
    if not args.no_prefill and world == 1:
        prefill.append(prefill_leg(rt, bank, stream, flush, 4096, args.seed, 10, 3, skew=False))
        prefill.append(prefill_leg(rt, bank, stream, flush, 8192, args.seed, 10, 3, skew=True))
    clocks.__exit__(None, None, None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_measure(T, args.seed)

    stack = None
    if world == 1 and not args.no_stack:
        # The headline line is printed whatever happens to this optional leg.
        try:
            stack = stack_leg(rt, args.seed, 30, 3, decode_kernels=args.decode_kernels)
        except Exception as error:  # noqa: BLE001
            stack = {"workload": "config4_stack40", "error": f"{type(error).__name__}: {error}"}

    linear = None
    if world == 1 and not args.no_linear:
        try:
            linear = linear_leg(rt, args.seed, 30, 3)
        except Exception as error:  # noqa: BLE001
            linear = {"workload": "lm_head_248320x2048", "error": f"{type(error).__name__}: {error}"}

    if rank == 0:
        clk = clocks.summary()
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 5),
            "ms_per_step_write_only_flush": round(wo_total_ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": ("nvfp4 weights x nvfp4 activations (four terms per row) on tcgen05, f32 accumulate; bf16 I/O"
                      if tc_decode else "nvfp4 weights x f16 activations, f32 accumulate; bf16 I/O"),
            "data": "synthetic (seeded BASELINE distributions; no checkpoint on this machine)",
            "config": {
                "workload": WORKLOAD,
                "tokens_per_step": T,
                "global_batch": T,
                "experts": E,
                "hidden": H,
                "intermediate": I,
                "top_k": 8,
                "shared_expert": True,
                "layers": 1,
                "parallelism": (f"ep{world}: {E // world} routed experts per GPU (shared expert on rank 0), "
                                "the 32 tokens replicated, combine fused with the cross-rank reduction over "
                                "NVLink peer memory" if world > 1 else "single GPU"),
                "l2": "flushed before every step (256 MiB write, then a 256 MiB read so no dirty line is "
                      "left) outside the per-step CUDA events",
                "inputs": f"pool of {pool_n} distinct token batches (the same on every rank)",
                "mean_unique_routed_experts": round(float(np.mean(uniq)), 2),
            },
            "us_per_token": round(1e6 / value, 4),
            "step_breakdown": breakdown,
            "layer_hbm_gbs": round(layer_bytes / (total_ms / 1000.0) / 1e9, 1),
            "decode_t1_us": ({"median": round(lat[len(lat) // 2], 3), "p10": round(lat[len(lat) // 10], 3),
                              "p90": round(lat[(9 * len(lat)) // 10], 3)} if lat else None),
            "kernels_ms_avg": {k: round(sum(v) / len(v), 5) for k, v in by_op.items()},
            "decode_t1_kernels_us": {k: round(statistics.median(v), 3) for k, v in t1_ops.items()},
            "roofline": {
                "kernel": "moe_gate_up",
                "bound": "hbm",
                "achieved": round(achieved, 1) if achieved else None,
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4) if achieved and peak else None,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (burst copy), of measured" if peak else "missing",
                "traffic": traffic,
                "algorithmic_bytes_per_launch": round(gu_bytes / max(1, len(gu))),
            },
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": 2 * T * H * 2 * world,
                    "d2h_bytes_per_step": T * H * 2 * world},
            "gpu_launches": launches * args.steps,
            "prefill": prefill,
            "expert_parallel": ep,
            "stack": stack,
            "linear": linear,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    bank.close()
    rt.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main() -> int:
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())
