"""CPU oracle for the NVFP4 MoE layer -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path, never the thing measured or
shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
leg of ``bench.py`` may import it. It restates, in plain numpy, the lab's
algorithm for the device-routed MoE bank of hotschmoe/x2-nvfp4-lab:

* NVFP4 decoding: E2M1 table ``native_nvfp4/kernels/nvfp4_gemv.cl:10-12``,
  E4M3 scale decoding ``nvfp4_gemv.cl:14-27`` and its numpy twin
  ``native_nvfp4/probe_native_nvfp4.py:121-130``, nibble order (low nibble =
  even column) ``nvfp4_gemv.cl:74-75``.
* NVFP4 GEMV: ``probe_native_nvfp4.py:133-141`` (``cpu_gemv``).
* Routing: top-8 by logit, lowest expert id on ties, weights
  ``exp(l_i - l_max) / sum_top8`` and slot 8 = (shared, sigmoid(shared
  logit)): ``nvfp4_gemv.cl:1249-1295``; host twin
  ``native_nvfp4/bench_moe_routed_layer.py:89-94``.
* Expert: ``bench_moe_routed_layer.py:97-103`` (gate, up, SiLU*up, down).
* Bank reduce and residual: ``nvfp4_gemv.cl:1443-1457`` and
  ``native_nvfp4/bench_moe_full_model.py:392-406``.

Extensions beyond the lab (which only decodes one token):
* batching and the dispatch permutation (histogram, offsets, stable
  token-ascending order within an expert);
* the BASELINE quantiser (the lab ships none): global g = amax/(6*448),
  block scale E4M3_RNE(blockamax/6/g), E2M1 round-to-nearest with ties to
  the even code;
* a bit-reproducible router dot product: BF16 weights times FP32/BF16
  activations accumulated in FP32 in the documented lane order used by the
  CUDA routing kernel.

Parity is pinned against golden vectors produced by running the reference's
own Python oracle functions (see ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

TOP_K = 8
FLT_MAX = np.float32(3.4028234663852886e38)

# E2M1 code -> value (nvfp4_gemv.cl:10-12).
E2M1 = np.asarray(
    [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32
)
_E2M1_MAG = E2M1[:8]


# ------------------------------------------------------------------ decoding


def decode_e4m3_scale(raw: np.ndarray) -> np.ndarray:
    """E4M3 scale byte -> float32 with the lab's rule: sign bit ignored,
    0x00 and 0x7F decode to 0, exponent 0 is subnormal m/512
    (nvfp4_gemv.cl:14-27, probe_native_nvfp4.py:121-127)."""
    raw = np.asarray(raw, dtype=np.uint8) & np.uint8(0x7F)
    exp = (raw >> np.uint8(3)).astype(np.int32)
    man = (raw & np.uint8(7)).astype(np.float64)
    out = np.where(exp == 0, man / 512.0, (1.0 + man / 8.0) * np.exp2(exp - 7.0))
    out = np.where((raw == 0) | (raw == 0x7F), 0.0, out)
    return out.astype(np.float32)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """[rows, cols/2] uint8 -> [rows, cols] float32 E2M1 values; the low nibble
    of byte b is column 2b (nvfp4_gemv.cl:74-75)."""
    packed = np.asarray(packed, dtype=np.uint8)
    rows, half = packed.shape
    out = np.empty((rows, half * 2), dtype=np.float32)
    out[:, 0::2] = E2M1[packed & 0x0F]
    out[:, 1::2] = E2M1[packed >> 4]
    return out


def dequantize(packed: np.ndarray, scales: np.ndarray, weight_global_scale: float) -> np.ndarray:
    """Dequantised float32 matrix: E2M1 * E4M3(scale) * (1/divisor). The
    divisor is inverted once in FP32, as the bank upload does
    (nvfp4_runtime.cpp:1895-1897)."""
    values = unpack_e2m1(packed)
    rows, cols = values.shape
    inv = np.float32(1.0) / np.float32(weight_global_scale)
    block = decode_e4m3_scale(scales).reshape(rows, cols // 16) * inv
    return (values.reshape(rows, cols // 16, 16) * block[:, :, None]).reshape(rows, cols)


def nvfp4_gemv(packed: np.ndarray, scales: np.ndarray, x: np.ndarray, weight_global_scale: float) -> np.ndarray:
    """Restatement of ``cpu_gemv`` (probe_native_nvfp4.py:133-141): per 16-block
    partial dot of E2M1 values with x in FP32, times the block scale divided
    by the global divisor, summed over blocks in FP32."""
    rows, half = packed.shape
    cols = half * 2
    blocks = cols // 16
    q = np.asarray(packed, dtype=np.uint8).reshape(rows, blocks, 8)
    xv = np.asarray(x, dtype=np.float32).reshape(blocks, 8, 2)
    local = decode_e4m3_scale(scales).reshape(rows, blocks) / np.float32(weight_global_scale)
    dots = E2M1[q & 0x0F] * xv[None, :, :, 0] + E2M1[q >> 4] * xv[None, :, :, 1]
    return np.sum(np.sum(dots, axis=2, dtype=np.float32) * local, axis=1, dtype=np.float32)


# ---------------------------------------------------------------- quantiser


def _e4m3_table() -> np.ndarray:
    codes = np.arange(0x7F, dtype=np.uint8)  # 0x00 .. 0x7E, monotonic values
    exp = (codes >> 3).astype(np.int32)
    man = (codes & 7).astype(np.float64)
    vals = np.where(exp == 0, man / 512.0, (1.0 + man / 8.0) * np.exp2(exp - 7.0))
    return vals


_E4M3_VALUES = _e4m3_table()


def e4m3_encode_rne(v: np.ndarray) -> np.ndarray:
    """Non-negative float -> E4M3 byte, round to nearest with ties to the even
    code, saturating at 448 (0x7E)."""
    v = np.minimum(np.asarray(v, dtype=np.float64), 448.0)
    hi = np.clip(np.searchsorted(_E4M3_VALUES, v, side="left"), 0, 0x7E)
    lo = np.clip(hi - 1, 0, 0x7E)
    dlo = v - _E4M3_VALUES[lo]
    dhi = _E4M3_VALUES[hi] - v
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    return np.where(pick_hi, hi, lo).astype(np.uint8)


def e2m1_encode_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> E2M1 code (4 bits), nearest magnitude on {0,.5,1,1.5,2,3,4,6},
    ties to the even code, saturating at 6; the sign bit follows signbit(x)."""
    x = np.asarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x).astype(np.float64), 6.0)
    hi = np.clip(np.searchsorted(_E2M1_MAG.astype(np.float64), mag, side="left"), 0, 7)
    lo = np.clip(hi - 1, 0, 7)
    dlo = mag - _E2M1_MAG[lo]
    dhi = _E2M1_MAG[hi] - mag
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return code | (np.signbit(x).astype(np.uint8) << 3)


@dataclass
class QuantizedMatrix:
    packed: np.ndarray       # [rows, cols/2] uint8
    scales: np.ndarray       # [rows, cols/16] uint8 (E4M3)
    global_scale: float      # the ABI divisor = 1/g


def quantize_nvfp4(w: np.ndarray) -> QuantizedMatrix:
    """BASELINE quantiser. g = amax/(6*448) in FP32; per 16-column block
    s = E4M3_RNE(blockamax/6/g); codes = E2M1_RNE(w / (s*g)) with the two FP32
    operations rounded separately. The ABI divisor is 1/g in FP32."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    amax = np.float32(np.max(np.abs(w))) if w.size else np.float32(0)
    g = np.float32(amax / np.float32(6.0 * 448.0)) if amax > 0 else np.float32(1.0)
    blocks = w.reshape(rows, cols // 16, 16)
    bamax = np.max(np.abs(blocks), axis=2)
    target = (bamax / np.float32(6.0)).astype(np.float32) / g
    scales = e4m3_encode_rne(target.astype(np.float32))
    s_val = decode_e4m3_scale(scales)
    denom = (s_val * g).astype(np.float32)
    safe = np.where(denom == 0, np.float32(1.0), denom)
    scaled = (blocks / safe[:, :, None]).astype(np.float32)
    scaled = np.where(denom[:, :, None] == 0, np.float32(0.0), scaled)
    codes = e2m1_encode_rne(scaled).reshape(rows, cols)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return QuantizedMatrix(packed, scales.reshape(rows, cols // 16), float(np.float32(1.0) / g))


# ------------------------------------------------------------------- BF16


def bf16_bits_from_f32(x: np.ndarray) -> np.ndarray:
    """float32 -> BF16 bits, round to nearest even (nvfp4_gemv.cl:46-50)."""
    bits = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ routing


def router_logits(router_bf16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """[T, R] float32 logits of BF16 rows [R, H] against x [T, H] (float32 or
    BF16-valued), in FP32 as the lab's bf16_gemv_subgroup accumulates
    (nvfp4_gemv.cl:1223-1247), with the CUDA routing kernel's fixed order:
    lane l (0..31) owns columns j*128 + 4l + e and adds (w*x rounded to FP32)
    to its FP32 sum with j then e ascending; the 32 lane sums then combine by
    an xor butterfly (16, 8, 4, 2, 1). Every operation is one IEEE FP32
    rounding, so the result is reproduced bit for bit."""
    w = bf16_bits_to_f32(router_bf16)
    x = np.asarray(x, dtype=np.float32)
    R, H = w.shape
    T = x.shape[0]
    assert H % 128 == 0
    wv = w.reshape(R, H // 128, 32, 4)
    xv = x.reshape(T, H // 128, 32, 4)
    acc = np.zeros((T, R, 32), dtype=np.float32)
    for j in range(H // 128):
        for e in range(4):
            prod = (xv[:, None, j, :, e] * wv[None, :, j, :, e]).astype(np.float32)
            acc = (acc + prod).astype(np.float32)
    for off in (16, 8, 4, 2, 1):
        idx = np.arange(32) ^ off
        acc = (acc + acc[:, :, idx]).astype(np.float32)
    return acc[:, :, 0].copy()


def top8_route(logits: np.ndarray, top_k: int = TOP_K) -> tuple[np.ndarray, np.ndarray]:
    """Top-k ids by descending logit, lowest id among equal logits, and the
    renormalised weights exp(l_i - l_0) / sum_j exp(l_j - l_0) in FP32
    (nvfp4_gemv.cl:1267-1290)."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    # Stable sort by (-logit, id): lexsort's last key is primary.
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -logits.astype(np.float64)), axis=1)
    ids = order[:, :top_k].astype(np.int32)
    top = np.take_along_axis(logits, ids, axis=1)
    ex = np.exp((top - top[:, :1]).astype(np.float32)).astype(np.float32)
    den = np.zeros(T, dtype=np.float32)
    for k in range(top_k):
        den = (den + ex[:, k]).astype(np.float32)
    weights = (ex / den[:, None]).astype(np.float32)
    return ids, weights


def sigmoid32(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


def dispatch(ids: np.ndarray, experts: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Histogram, exclusive offsets and the stable dispatch permutation: flat
    (token*k + slot) indices grouped by expert ascending, token ascending
    within an expert."""
    ids = np.asarray(ids, dtype=np.int64)
    T, K = ids.shape
    flat = ids.reshape(-1)
    counts = np.bincount(flat, minlength=experts).astype(np.int32)
    offsets = np.zeros(experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    perm = np.argsort(flat, kind="stable").astype(np.int32)
    return counts, offsets, perm


# --------------------------------------------------------------------- bank


@dataclass
class BankHost:
    """Host copy of a bank: projections[p][expert] = QuantizedMatrix, with
    expert index `experts` the shared expert; router [E, H] and shared gate
    [H] as BF16 bits; optional FP32 router bias [E]."""

    experts: int
    hidden: int
    intermediate: int
    router_bf16: np.ndarray
    shared_gate_bf16: np.ndarray
    projections: list[dict[int, QuantizedMatrix]] = field(default_factory=lambda: [{}, {}, {}])
    router_bias: np.ndarray | None = None
    _dequant: dict = field(default_factory=dict)

    def weight(self, expert: int, projection: int) -> np.ndarray:
        key = (expert, projection)
        if key not in self._dequant:
            m = self.projections[projection][expert]
            self._dequant[key] = dequantize(m.packed, m.scales, m.global_scale)
        return self._dequant[key]

    def router_all(self) -> np.ndarray:
        return np.concatenate([self.router_bf16, self.shared_gate_bf16.reshape(1, -1)], axis=0)


def expert_forward(bank: BankHost, expert: int, x: np.ndarray) -> np.ndarray:
    """SwiGLU expert on dequantised FP32 weights, FP64 matmuls
    (bench_moe_routed_layer.py:97-103). x [n, H] -> [n, H]."""
    x = np.asarray(x, dtype=np.float64)
    gate = x @ bank.weight(expert, 0).astype(np.float64).T
    up = x @ bank.weight(expert, 1).astype(np.float64).T
    act = gate / (1.0 + np.exp(-gate)) * up
    return act @ bank.weight(expert, 2).astype(np.float64).T


@dataclass
class LayerResult:
    out: np.ndarray          # [T, H] float64 (before any output rounding)
    logits: np.ndarray       # [T, E+1] float32
    ids: np.ndarray          # [T, 9] int32 (slot 8 = shared expert id E)
    weights: np.ndarray      # [T, 9] float32 (slot 8 = sigmoid)
    counts: np.ndarray
    offsets: np.ndarray
    perm: np.ndarray


def moe_layer(bank: BankHost, x: np.ndarray, residual: np.ndarray | None = None,
              expert_range: tuple[int, int] | None = None, shared_here: bool = True) -> LayerResult:
    """Full layer: router -> top-8 -> dispatch -> routed + shared SwiGLU experts
    -> weighted combine (+ residual). x is [T, H] float32 (BF16 values are
    passed as their float32 images).

    With ``expert_range = (first, count)`` the output is the partial sum of an
    expert-parallel rank: only routed experts in [first, first + count) are
    added, the shared expert only when ``shared_here`` (routing is unchanged)."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    E = bank.experts
    logits = router_logits(bank.router_all(), x)
    if bank.router_bias is not None:
        logits[:, :E] = (logits[:, :E] + np.asarray(bank.router_bias, dtype=np.float32)).astype(np.float32)
    ids, weights = top8_route(logits[:, :E])
    shared_w = sigmoid32(logits[:, E])
    counts, offsets, perm = dispatch(ids, E)
    out = np.zeros((T, H), dtype=np.float64)
    first, count = expert_range if expert_range is not None else (0, E)
    for e in np.unique(ids):
        if not first <= int(e) < first + count:
            continue
        rows, slots = np.nonzero(ids == e)
        y = expert_forward(bank, int(e), x[rows])
        out[rows] += weights[rows, slots].astype(np.float64)[:, None] * y
    if shared_here:
        out += shared_w.astype(np.float64)[:, None] * expert_forward(bank, E, x)
    if residual is not None:
        out += np.asarray(residual, dtype=np.float64)
    ids9 = np.concatenate([ids, np.full((T, 1), E, dtype=np.int32)], axis=1)
    w9 = np.concatenate([weights, shared_w[:, None]], axis=1).astype(np.float32)
    return LayerResult(out, logits, ids9, w9, counts, offsets, perm)


# ------------------------------------------------- prefill activation terms


@dataclass
class RowTerms:
    codes: np.ndarray        # [terms, rows, cols/2] uint8 (low nibble = even column)
    words: np.ndarray        # [terms, rows, cols/64] uint32 (four E4M3 block scales, low byte first)
    g: np.ndarray            # [rows] float32
    approx: np.ndarray       # [rows, cols] float32: sum of the dequantised terms


def quantize_rows_split(x: np.ndarray, terms: int) -> RowTerms:
    """The prefill path's activation quantiser (this library's definition;
    the lab quantises no activations). Per row g = amax/2688 in FP32 (1 for
    an all-zero row); per term and 16-column block of the remainder r:
    s = E4M3_RNE((bamax/6)/g), d = s*g, code = E2M1_RNE(r * RN(1/d)) with a
    zero magnitude always unsigned (0 when d is 0), r -= code*d -- every
    operation rounded to FP32 separately, as the CUDA kernel does."""
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    f32 = np.float32
    amax = np.max(np.abs(x), axis=1).astype(f32)
    g = np.where(amax > 0, (amax / f32(2688.0)).astype(f32), f32(1.0)).astype(f32)
    r = x.reshape(rows, cols // 16, 16).copy()
    approx = np.zeros_like(r)
    codes_all, words_all = [], []
    for _ in range(terms):
        bamax = np.max(np.abs(r), axis=2).astype(f32)
        target = ((bamax / f32(6.0)).astype(f32) / g[:, None]).astype(f32)
        s = e4m3_encode_rne(target)
        denom = (decode_e4m3_scale(s).astype(f32) * g[:, None]).astype(f32)
        with np.errstate(divide="ignore"):
            inv = np.where(denom != 0, (f32(1.0) / denom).astype(f32), f32(0.0)).astype(f32)
        q = (r * inv[:, :, None]).astype(f32)
        codes = e2m1_encode_rne(q)
        codes = np.where((codes & 7) == 0, 0, codes).astype(np.uint8)
        deq = (E2M1[codes] * denom[:, :, None]).astype(f32)
        approx = (approx + deq).astype(f32)
        r = (r - deq).astype(f32)
        flat = codes.reshape(rows, cols)
        codes_all.append((flat[:, 0::2] | (flat[:, 1::2] << 4)).astype(np.uint8))
        sb = s.reshape(rows, cols // 64, 4).astype(np.uint32)
        words_all.append(sb[..., 0] | (sb[..., 1] << 8) | (sb[..., 2] << 16) | (sb[..., 3] << 24))
    # approx is accumulated in term order; the GEMM sums exact products of
    # the terms, so this is the value it multiplies.
    return RowTerms(np.stack(codes_all), np.stack(words_all).astype(np.uint32), g,
                    approx.reshape(rows, cols))


def dequantize_terms(t: RowTerms) -> np.ndarray:
    """Sum of the dequantised terms in float64 (what the tensor cores add)."""
    terms, rows, half = t.codes.shape
    cols = half * 2
    total = np.zeros((rows, cols), dtype=np.float64)
    for j in range(terms):
        c = np.empty((rows, cols), dtype=np.uint8)
        c[:, 0::2] = t.codes[j] & 0xF
        c[:, 1::2] = t.codes[j] >> 4
        sb = np.stack([(t.words[j] >> (8 * b)) & 0xFF for b in range(4)], axis=-1).reshape(rows, cols // 16)
        sv = decode_e4m3_scale(sb.astype(np.uint8)).astype(np.float64)
        total += E2M1[c].astype(np.float64) * np.repeat(sv, 16, axis=1) * t.g.astype(np.float64)[:, None]
    return total


def moe_layer_prefill(bank: BankHost, x: np.ndarray, residual: np.ndarray | None = None,
                      x_terms: int = 4, act_terms: int = 3) -> LayerResult:
    """The layer as the prefill path computes it: routing exactly as
    moe_layer; expert inputs replaced by their x_terms NVFP4 terms;
    SiLU(gate)*up rounded to FP16 and replaced by its act_terms terms before
    the down projection; products and sums in float64."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    E = bank.experts
    logits = router_logits(bank.router_all(), x)
    if bank.router_bias is not None:
        logits[:, :E] = (logits[:, :E] + np.asarray(bank.router_bias, dtype=np.float32)).astype(np.float32)
    ids, weights = top8_route(logits[:, :E])
    shared_w = sigmoid32(logits[:, E])
    counts, offsets, perm = dispatch(ids, E)
    xq = dequantize_terms(quantize_rows_split(x, x_terms))

    def expert(e: int, rows: np.ndarray) -> np.ndarray:
        xin = xq[rows]
        gate = xin @ bank.weight(e, 0).astype(np.float64).T
        up = xin @ bank.weight(e, 1).astype(np.float64).T
        act = (gate / (1.0 + np.exp(-gate)) * up).astype(np.float32).astype(np.float16).astype(np.float32)
        aq = dequantize_terms(quantize_rows_split(act, act_terms))
        return aq @ bank.weight(e, 2).astype(np.float64).T

    out = np.zeros((T, H), dtype=np.float64)
    for e in np.unique(ids):
        rows, slots = np.nonzero(ids == e)
        out[rows] += weights[rows, slots].astype(np.float64)[:, None] * expert(int(e), rows)
    out += shared_w.astype(np.float64)[:, None] * expert(E, np.arange(T))
    if residual is not None:
        out += np.asarray(residual, dtype=np.float64)
    ids9 = np.concatenate([ids, np.full((T, 1), E, dtype=np.int32)], axis=1)
    w9 = np.concatenate([weights, shared_w[:, None]], axis=1).astype(np.float32)
    return LayerResult(out, logits, ids9, w9, counts, offsets, perm)


# ------------------------------------------------------------- comparisons


def rmsnorm_bf16(x: np.ndarray, weight: np.ndarray | None = None, epsilon: float = 1e-6) -> np.ndarray:
    """Row-wise RMSNorm of x [rows, cols] (BF16 values held in FP32), output
    rounded to BF16 values. The lab's ``rmsnorm_f32``
    (``native_nvfp4/kernels/nvfp4_gemv.cl:1171-1197``: sum of squares,
    x * rsqrt(mean + epsilon) * weight) in the reduction order of the CUDA
    kernel that serves it: 256 column-strided FP32 partial sums (fused
    multiply-add), an xor butterfly over each warp of 32 partials (offsets
    16, 8, 4, 2, 1), the eight warp sums added in order from 0. The CUDA
    kernel's rsqrtf is within 2 ulp of the 1/sqrt used here."""
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    w = np.ones(cols, dtype=np.float32) if weight is None else np.asarray(weight, dtype=np.float32)
    threads = 256
    part = np.zeros((rows, threads), dtype=np.float32)
    for c0 in range(0, cols, threads):
        v = x[:, c0:c0 + threads].astype(np.float64)
        n = v.shape[1]
        # fmaf(v, v, ss): the exact v*v + ss rounded once to FP32.
        part[:, :n] = (v * v + part[:, :n].astype(np.float64)).astype(np.float32)
    warps = part.reshape(rows, threads // 32, 32)
    for off in (16, 8, 4, 2, 1):
        idx = np.arange(32) ^ off
        warps = (warps + warps[:, :, idx]).astype(np.float32)
    tot = np.zeros(rows, dtype=np.float32)
    for wi in range(threads // 32):
        tot = (tot + warps[:, wi, 0]).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(tot / np.float32(cols) + np.float32(epsilon))).astype(np.float32)
    out = ((x * inv[:, None]).astype(np.float32) * w[None, :]).astype(np.float32)
    return bf16_bits_to_f32(bf16_bits_from_f32(out))


def moe_stack(banks: list[BankHost], x: np.ndarray, epsilon: float = 1e-6, norm_weights=None) -> np.ndarray:
    """Resident decode stack without attention, BF16 hidden state: per layer
    h = BF16(h + moe_layer(RMSNorm(h))), the lab's full-model step
    (``native_nvfp4/bench_moe_full_model.py:388-406``: ``rmsnorm_device``,
    ``bank.decode_device``, ``add_device``) with its attention omitted."""
    h = bf16_bits_to_f32(bf16_bits_from_f32(np.asarray(x, dtype=np.float32)))
    for layer, bank in enumerate(banks):
        w = None if norm_weights is None else norm_weights[layer]
        normed = rmsnorm_bf16(h, w, epsilon)
        h = bf16_bits_to_f32(bf16_bits_from_f32(moe_layer(bank, normed, h).out))
    return h


def rel_rmse(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = np.sqrt(np.mean(e * e))
    return float(np.sqrt(np.mean((a - e) ** 2)) / den) if den > 0 else float(np.sqrt(np.mean(a * a)))


def max_abs_rel(actual: np.ndarray, expected: np.ndarray) -> float:
    """max |a - e| / max |e| (the BASELINE max-abs-relative criterion)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = np.max(np.abs(e))
    return float(np.max(np.abs(a - e)) / den) if den > 0 else float(np.max(np.abs(a)))
