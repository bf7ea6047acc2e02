"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference's OWN Python oracle functions, imported unchanged from a
checkout of hotschmoe/x2-nvfp4-lab, on seeded synthetic inputs and stores
inputs and outputs as small .npz fixtures next to this script:

* ``decode_e4m3_scale`` and ``E2M1`` -- native_nvfp4/probe_native_nvfp4.py:121-130
* ``cpu_gemv``                       -- native_nvfp4/probe_native_nvfp4.py:133-141
* ``route``                          -- native_nvfp4/bench_moe_routed_layer.py:89-94
* ``expert_reference``               -- native_nvfp4/bench_moe_routed_layer.py:97-103
* the single-token layer composition of
  native_nvfp4/bench_moe_device_bank.py:107-120 (route on the FP32 router
  logits, weighted routed experts plus the sigmoid-gated shared expert).

Run where the reference checkout exists:
    python tests/golden/make_golden.py --reference <path to x2-nvfp4-lab>
The tests only read the .npz files; they never need the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import synthetic_np  # noqa: E402
from oracle.nvfp4_oracle import bf16_bits_to_f32, quantize_nvfp4  # noqa: E402


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "native_nvfp4"))
    import bench_moe_routed_layer as ref_layer  # noqa: E402
    import probe_native_nvfp4 as ref_probe  # noqa: E402

    rng = np.random.default_rng(20260822)

    # 1. E4M3 scale decoding table and E2M1 values.
    all_bytes = np.arange(256, dtype=np.uint8)
    np.savez_compressed(
        HERE / "golden_decode.npz",
        e4m3=ref_probe.decode_e4m3_scale(all_bytes.copy()),
        e2m1=np.asarray(ref_probe.E2M1, dtype=np.float32),
    )

    # 2. NVFP4 GEMV on random packed bytes and scale bytes (every byte value).
    gemv = {}
    for i, (rows, cols, divisor) in enumerate([(16, 64, 1.0), (64, 256, 37.5), (256, 1024, 2688.0 / 0.1),
                                               (1024, 256, 913.25)]):
        packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        scales = rng.integers(0, 256, (rows, cols // 16), dtype=np.uint8)
        x = (rng.standard_normal(cols).astype(np.float32) * np.float32(0.2)).astype(np.float32)
        gemv[f"packed{i}"] = packed
        gemv[f"scales{i}"] = scales
        gemv[f"x{i}"] = x
        gemv[f"divisor{i}"] = np.float32(divisor)
        gemv[f"out{i}"] = ref_probe.cpu_gemv(packed, scales, x, divisor)
    np.savez_compressed(HERE / "golden_gemv.npz", **gemv)

    # 3. Routing of 256-expert logits (no exact ties; torch.topk's tie order
    #    is unspecified, so tie cases are pinned by the oracle's own tests).
    logits = (rng.standard_normal((64, 256)).astype(np.float32) * np.float32(0.9)).astype(np.float32)
    ids = np.zeros((64, 8), dtype=np.int32)
    weights = np.zeros((64, 8), dtype=np.float32)
    for t in range(64):
        sel, w = ref_layer.route(logits[t], 8)
        ids[t] = sel
        weights[t] = w
    np.savez_compressed(HERE / "golden_route.npz", logits=logits, ids=ids, weights=weights)

    # 4. One SwiGLU expert (H=256, I=128) on four tokens.
    H, I = 256, 128
    proj = []
    arrays = {}
    for p, shape in enumerate([(I, H), (I, H), (H, I)]):
        q = quantize_nvfp4(rng.standard_normal(shape).astype(np.float32) * np.float32(0.02))
        proj.append((q.packed, q.scales, q.global_scale))
        arrays[f"packed{p}"] = q.packed
        arrays[f"scales{p}"] = q.scales
        arrays[f"divisor{p}"] = np.float32(q.global_scale)
    xe = bf16_bits_to_f32(synthetic_np.tokens_bf16(4, H, 7))
    arrays["x"] = xe
    arrays["out"] = ref_layer.expert_reference(proj, xe)
    np.savez_compressed(HERE / "golden_expert.npz", **arrays)

    # 5. Single-token layers composed as bench_moe_device_bank.py:107-120 does,
    #    on seeded synthetic banks (weights regenerated from seeds by the test;
    #    the hashes guard against generator drift).
    layers = {}
    for name, (E, H, I, seed, T) in {
        "small": (16, 256, 128, 11, 4),
        "config0": (256, 2048, 512, 0, 1),
    }.items():
        router = synthetic_np.router_bf16(E, H, seed)
        gate = synthetic_np.shared_gate_bf16(H, seed)
        xs = bf16_bits_to_f32(synthetic_np.tokens_bf16(T, H, seed))
        router_f32 = bf16_bits_to_f32(router)
        gate_f32 = bf16_bits_to_f32(gate)
        outs, all_ids, all_w, shared_logits, hashes = [], [], [], [], []
        cache = {}

        def expert(e: int):
            if e not in cache:
                cache[e] = [synthetic_np.expert_projection(e, p, H, I, seed) for p in range(3)]
            return [(q.packed, q.scales, q.global_scale) for q in cache[e]]

        for t in range(T):
            x = xs[t : t + 1]
            sel, w = ref_layer.route(router_f32 @ x[0], 8)
            shared_logit = float((gate_f32 @ x[0]).item())
            shared_weight = float(1.0 / (1.0 + np.exp(-shared_logit)))
            ref = np.zeros((1, H), dtype=np.float32)
            for wt, e in zip(w, sel, strict=True):
                ref += np.float32(wt) * ref_layer.expert_reference(expert(int(e)), x)
            ref += np.float32(shared_weight) * ref_layer.expert_reference(expert(E), x)
            outs.append(ref[0])
            all_ids.append(np.asarray(sel, dtype=np.int32))
            all_w.append(np.asarray(w, dtype=np.float32))
            shared_logits.append(shared_logit)
        for e in sorted(cache):
            hashes.append(f"{e}:" + sha(*[a for q in cache[e] for a in (q.packed, q.scales)]))
        layers[f"{name}_shape"] = np.asarray([E, H, I, seed, T], dtype=np.int64)
        layers[f"{name}_out"] = np.stack(outs)
        layers[f"{name}_ids"] = np.stack(all_ids)
        layers[f"{name}_weights"] = np.stack(all_w)
        layers[f"{name}_shared_logit"] = np.asarray(shared_logits, dtype=np.float64)
        layers[f"{name}_hashes"] = np.asarray(hashes)
    np.savez_compressed(HERE / "golden_layer.npz", **layers)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
