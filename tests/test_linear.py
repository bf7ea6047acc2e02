"""Dense NVFP4 linear (the lab's nvfp4_matrix / nvfp4_linear_* entry points and
its vLLM NvFp4LinearKernel provider).

CPU: the provider's contract with a fake runtime (what it uploads, how it
reshapes, casts and adds the bias) and its registration. GPU (sm_100a): every
linear entry point (the tensor-core kernel; the CUDA-core kernel for the scalar
kernel kind) against the oracle's restatement of the lab's CPU GEMV
(``nvfp4_gemv``, pinned to the lab's golden vectors), at the lab's own GEMV
gate (2e-5 of the output scale), including ragged shapes, several passes of
vectors, and scale bytes outside the E4M3 value range (sign bit, 0x7F)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.nvfp4_oracle import E2M1 as _E2M1
from oracle.nvfp4_oracle import decode_e4m3_scale as _decode_e4m3_scale
from oracle.nvfp4_oracle import nvfp4_gemv

GATE = 2e-5  # probe_native_nvfp4.py:294


def _oracle(packed, scales, x, divisor):
    return np.stack([nvfp4_gemv(packed, scales, x[v], divisor) for v in range(x.shape[0])])


def _matrix(rows, cols, seed, full_scale_bytes=False):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    if full_scale_bytes:
        scales = rng.integers(0, 256, size=(rows, cols // 16), dtype=np.uint8)
    else:
        scales = rng.integers(0x30, 0x48, size=(rows, cols // 16), dtype=np.uint8)  # 2^-1 .. 2^2
    return packed, scales


# ------------------------------------------------------------------ CPU


class _FakeRuntime:
    def __init__(self):
        self.uploaded = None
        self.calls = []

    def upload(self, packed, scales, divisor):
        from vllm_nvfp4_cuda.runtime import NativeMatrix

        self.uploaded = (packed, scales, divisor)
        m = NativeMatrix.__new__(NativeMatrix)
        m.runtime, m.handle, m.rows, m.cols, m.shared_svm = None, None, packed.shape[0], packed.shape[1] * 2, False
        return m

    def linear_tensor(self, matrix, x):
        import torch

        self.calls.append((x.dtype, tuple(x.shape)))
        packed, scales, divisor = self.uploaded
        flat = x.reshape(-1, matrix.cols).numpy()
        out = _oracle(packed, scales, flat, divisor)
        return torch.from_numpy(out).reshape(*x.shape[:-1], matrix.rows)


def test_provider_contract_with_fake_runtime(monkeypatch):
    import torch

    import vllm_nvfp4_cuda.linear as provider
    from vllm.model_executor.kernels.linear.nvfp4 import NvFp4LinearLayerConfig

    with pytest.raises(RuntimeError, match="requires CUDA activations"):
        provider._require_cuda(torch.zeros(1, 16))
    fake = _FakeRuntime()
    monkeypatch.setattr(provider, "get_runtime", lambda: fake)
    monkeypatch.setattr(provider, "_require_cuda", lambda x: None)  # the fake computes on the CPU
    monkeypatch.setattr(provider, "provider_enabled", lambda: (True, None))
    rows, cols = 48, 64
    packed, scales = _matrix(rows, cols, 3)
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(torch.from_numpy(packed.copy()), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(torch.from_numpy(scales.copy()).view(torch.float8_e4m3fn),
                                            requires_grad=False)
    layer.weight_global_scale = torch.nn.Parameter(torch.tensor(4.0), requires_grad=False)
    kernel = provider.CudaNvFp4LinearKernel(NvFp4LinearLayerConfig())
    assert provider.CudaNvFp4LinearKernel.supports_a16()
    assert provider.CudaNvFp4LinearKernel.is_supported(90)[0] is False
    kernel.process_weights_after_loading(layer)
    up_packed, up_scales, divisor = fake.uploaded
    np.testing.assert_array_equal(up_packed, packed)
    np.testing.assert_array_equal(up_scales, scales)
    assert divisor == 0.25  # the inverse of weight_global_scale, as the lab passes it

    x = torch.randn(2, 3, cols, dtype=torch.bfloat16)
    bias = torch.randn(rows, dtype=torch.bfloat16)
    y = kernel.apply_weights(layer, x, bias)
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (2, 3, rows)
    assert fake.calls == [(torch.float32, (2, 3, cols))]
    ref = _oracle(packed, scales, x.float().reshape(-1, cols).numpy(), 0.25).reshape(2, 3, rows)
    expect = torch.from_numpy(ref).to(torch.bfloat16) + bias
    assert torch.equal(y, expect)
    with pytest.raises(ValueError, match="does not match matrix width"):
        kernel.apply_weights(layer, torch.zeros(1, cols + 16))


def test_register_adds_cuda_linear_provider():
    import vllm_nvfp4_cuda
    from vllm.model_executor.kernels import linear as kl

    from vllm.platforms import PlatformEnum

    vllm_nvfp4_cuda.register()
    vllm_nvfp4_cuda.register()  # idempotent
    from vllm_nvfp4_cuda.linear import CudaNvFp4LinearKernel

    assert kl._POSSIBLE_NVFP4_KERNELS[PlatformEnum.CUDA].count(CudaNvFp4LinearKernel) == 1


def test_gemv_oracle_handles_ragged_columns():
    """cols a multiple of 16 but not of 32: the oracle agrees with the
    dequantise-then-matmul form (the GPU tests rely on it at such widths)."""
    from oracle.nvfp4_oracle import dequantize

    packed, scales = _matrix(7, 48, 5, full_scale_bytes=True)
    x = np.random.default_rng(6).standard_normal(48).astype(np.float32)
    dense = dequantize(packed, scales, 3.0).astype(np.float64) @ x.astype(np.float64)
    got = nvfp4_gemv(packed, scales, x, 3.0)
    np.testing.assert_allclose(got, dense, rtol=1e-5, atol=1e-5 * np.max(np.abs(dense)))


def _emulate_kernel(packed, scales, x, divisor, grid, V=4):
    """The launch plan of nvfp4_linear_kernel<V> (csrc/linear.cu) run on the CPU:
    the upload's pitches and scale sanitising, the rotated shared-memory slots
    of the activations (every slot written once, nothing read unwritten), each
    lane's chunks of each warp's four rows, two chunks per lane loaded
    together (16-byte packed words, two scale bytes, low nibble = even
    column; a chunk past the row re-reads the last one and is skipped), and
    the row loop over the grid (every output written once)."""
    RPW, CIF = 4, 2  # rows per warp, chunks in flight per lane (csrc/linear.cu)
    rows, half = packed.shape; cols = half * 2
    pp = (half + 15) // 16 * 16; sp = (cols // 16 + 15) // 16 * 16
    P = np.zeros((rows, pp), np.uint8); P[:, :half] = packed
    S = np.zeros((rows, sp), np.uint8); s = scales & 0x7F; s[s == 0x7F] = 0; S[:, :cols // 16] = s
    chunks = pp // 16; xcols = chunks * 32; vectors = x.shape[0]
    def xs_index(v, col):
        c, g, e = col >> 5, (col >> 2) & 7, col & 3
        return (v * chunks + c) * 32 + (((g + c) & 7) << 2) + e
    dst = np.full((vectors, rows), np.nan, np.float32)
    for v0 in range(0, vectors, V):
        xs = np.full(V * xcols, np.nan, np.float32); seen = set()
        for i in range(V * xcols):
            v, col = divmod(i, xcols); gv = v0 + v
            idx = xs_index(v, col); assert idx not in seen and 0 <= idx < V * xcols; seen.add(idx)
            xs[idx] = x[gv, col] if (gv < vectors and col < cols) else 0.0
        for b in range(grid):
            for w in range(8):
                r0 = (b * 8 + w) * RPW
                while r0 < rows:
                    acc = np.zeros((RPW, V, 32), np.float32)
                    for lane in range(32):
                        loaded = [min(cb + 32 * u, chunks - 1) for cb in range(lane, chunks, 32 * CIF)
                                  for u in range(CIF)]
                        used = [cb + 32 * u for cb in range(lane, chunks, 32 * CIF) for u in range(CIF)
                                if cb + 32 * u < chunks]
                        assert all(0 <= c < chunks for c in loaded)
                        assert used == list(range(lane, chunks, 32))
                        for c in used:
                            for j in range(RPW):
                                r = min(r0 + j, rows - 1)
                                q = P[r, c * 16:c * 16 + 16]
                                sc = _decode_e4m3_scale(S[r, c * 2:c * 2 + 2])
                                for wi in range(4):
                                    word = q[wi * 4:wi * 4 + 4]
                                    s2 = sc[0] if wi < 2 else sc[1]
                                    wv = np.empty(8, np.float32)
                                    for k in range(4):
                                        wv[2 * k] = _E2M1[word[k] & 15] * s2
                                        wv[2 * k + 1] = _E2M1[word[k] >> 4] * s2
                                    col = c * 32 + wi * 8
                                    for v in range(V):
                                        xv = np.array([xs[xs_index(v, col + t)] for t in range(8)], np.float32)
                                        acc[j, v, lane] += np.float32(np.dot(wv.astype(np.float64), xv.astype(np.float64)))
                    for j in range(RPW):
                        for v in range(V):
                            r, gv = r0 + j, v0 + v
                            if r < rows and gv < vectors:
                                assert np.isnan(dst[gv, r]); dst[gv, r] = acc[j, v].sum() / np.float32(divisor)
                    r0 += grid * 8 * RPW
    return dst


@pytest.mark.parametrize("rows,cols,vectors,grid", [(37, 48, 3, 2), (70, 1056, 5, 1), (5, 16, 1, 4)])
def test_kernel_launch_plan_on_cpu(rows, cols, vectors, grid):
    rng = np.random.default_rng(rows + cols)
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(0, 256, (rows, cols // 16), dtype=np.uint8)
    x = rng.standard_normal((vectors, cols)).astype(np.float32)
    got = _emulate_kernel(packed, scales, x, 2.0, grid)
    ref = _oracle(packed, scales, x, 2.0)
    assert not np.isnan(got).any()
    np.testing.assert_allclose(got, ref, rtol=GATE, atol=GATE * float(np.max(np.abs(ref))))


# ------------------------------------------------------------------ GPU

SHAPES = [  # (rows, cols, vectors)
    (1000, 2048, 1),
    (257, 528, 3),     # cols % 32 == 16: the last chunk is half padding
    (64, 16, 2),       # one block per row
    (33, 4096, 9),     # two passes (8 + 1 vectors)
    (4099, 1024, 4),
]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,vectors", SHAPES)
def test_linear_matches_oracle(cuda_runtime, rows, cols, vectors):
    packed, scales = _matrix(rows, cols, rows + cols)
    x = np.random.default_rng(vectors).standard_normal((vectors, cols)).astype(np.float32)
    divisor = 2.5
    m = cuda_runtime.upload(packed, scales, divisor)
    try:
        got = cuda_runtime.linear(m, x)
        ref = _oracle(packed, scales, x, divisor)
        np.testing.assert_allclose(got, ref, rtol=GATE, atol=GATE * float(np.max(np.abs(ref))))
    finally:
        m.close()


@pytest.mark.gpu
def test_linear_activation_range(cuda_runtime):
    """Each vector's activations enter as NVFP4 terms under the vector's own
    FP32 global scale: vectors far above and below FP16 range, one mixing a
    few large entries with ordinary ones, and a zero vector all meet the
    lab's gate, each relative to its own output scale."""
    rows, cols = 200, 1024
    packed, scales = _matrix(rows, cols, 41)
    x = np.random.default_rng(42).standard_normal((5, cols)).astype(np.float32)
    x[0] *= np.float32(1e6)
    x[1] *= np.float32(1e-30)
    x[2, :10] *= np.float32(1e5)
    x[3] = 0.0
    x[4] *= np.float32(3e-5)  # below FP16's smallest normal before scaling
    m = cuda_runtime.upload(packed, scales, 2.0)
    try:
        got = cuda_runtime.linear(m, x)
        ref = _oracle(packed, scales, x, 2.0)
        for v in range(x.shape[0]):
            scale = float(np.max(np.abs(ref[v])))
            np.testing.assert_allclose(got[v], ref[v], rtol=GATE, atol=GATE * scale, err_msg=f"vector {v}")
        assert not np.any(got[3])
    finally:
        m.close()


@pytest.mark.gpu
def test_linear_scale_bytes_follow_the_lab_rule(cuda_runtime):
    packed, scales = _matrix(300, 512, 11, full_scale_bytes=True)
    scales[:, 0] = 0x7F
    scales[:, 1] = 0xFF
    scales[:, 2] = 0xB8  # sign bit set: decoded as +1.0
    x = np.random.default_rng(12).standard_normal((2, 512)).astype(np.float32)
    m = cuda_runtime.upload(packed, scales, 1.0)
    try:
        got = cuda_runtime.linear(m, x)
        ref = _oracle(packed, scales, x, 1.0)
        np.testing.assert_allclose(got, ref, rtol=GATE, atol=GATE * float(np.max(np.abs(ref))))
    finally:
        m.close()


@pytest.mark.gpu
def test_linear_entry_points_agree(cuda_runtime):
    """Host, device-buffer, enqueued and tensor entry points run the same
    tensor-core kernel: bit-identical outputs. The scalar kernel kind runs
    the CUDA-core kernel on the FP32 activations: within the lab's gate of
    the tensor-core result and of the oracle."""
    import torch

    from vllm_nvfp4_cuda.runtime import KERNEL_SCALAR, KERNEL_SUBGROUP, KERNEL_TILED

    rows, cols, vectors = 515, 768, 5
    packed, scales = _matrix(rows, cols, 21)
    x = np.random.default_rng(22).standard_normal((vectors, cols)).astype(np.float32)
    m = cuda_runtime.upload(packed, scales, 6.0)
    try:
        host = cuda_runtime.linear(m, x, kernel_kind=KERNEL_TILED)
        xb = cuda_runtime.upload_buffer(x)
        ob = cuda_runtime.create_buffer(vectors * rows * 4)
        cuda_runtime.linear_device(m, xb, vectors, ob, kernel_kind=KERNEL_SUBGROUP)
        np.testing.assert_array_equal(ob.download((vectors, rows)), host)
        ob2 = cuda_runtime.create_buffer(vectors * rows * 4)
        cuda_runtime.linear_device(m, xb, vectors, ob2, kernel_kind=KERNEL_TILED, enqueue=True)
        cuda_runtime.synchronize()
        np.testing.assert_array_equal(ob2.download((vectors, rows)), host)
        xt = torch.from_numpy(x).cuda().reshape(1, vectors, cols)
        yt = cuda_runtime.linear_tensor(m, xt)
        torch.cuda.synchronize()
        assert tuple(yt.shape) == (1, vectors, rows)
        np.testing.assert_array_equal(yt.cpu().numpy().reshape(vectors, rows), host)
        ob3 = cuda_runtime.create_buffer(vectors * rows * 4)
        cuda_runtime.linear_device(m, xb, vectors, ob3, kernel_kind=KERNEL_SCALAR)
        scalar = ob3.download((vectors, rows))
        ref = _oracle(packed, scales, x, 6.0)
        for got in (scalar, host):
            np.testing.assert_allclose(got, ref, rtol=GATE, atol=GATE * float(np.max(np.abs(ref))))
        for b in (xb, ob, ob2, ob3):
            b.close()
    finally:
        m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("vectors", [21, 22, 43])
def test_linear_tensor_core_passes(cuda_runtime, vectors):
    """The tensor-core kernel carries 21 vectors per pass (six activation
    terms each in one 128-row B tile): full, one-over and two-over passes."""
    rows, cols = 700, 1280
    packed, scales = _matrix(rows, cols, 31 + vectors)
    x = np.random.default_rng(vectors).standard_normal((vectors, cols)).astype(np.float32)
    m = cuda_runtime.upload(packed, scales, 3.0)
    try:
        got = cuda_runtime.linear(m, x)
        ref = _oracle(packed, scales, x, 3.0)
        np.testing.assert_allclose(got, ref, rtol=GATE, atol=GATE * float(np.max(np.abs(ref))))
    finally:
        m.close()


@pytest.mark.gpu
def test_linear_argument_errors(cuda_runtime):
    from vllm_nvfp4_cuda.runtime import KERNEL_ROW_TILED, KERNEL_TILED

    packed, scales = _matrix(32, 64, 31)
    m = cuda_runtime.upload(packed, scales, 1.0)
    try:
        with pytest.raises(RuntimeError, match="tiled kernel requires more than one vector"):
            cuda_runtime.linear(m, np.zeros((1, 64), np.float32), kernel_kind=KERNEL_TILED)
        with pytest.raises(RuntimeError, match="row-tiled kernel requires one vector"):
            cuda_runtime.linear(m, np.zeros((2, 64), np.float32), kernel_kind=KERNEL_ROW_TILED)
        with pytest.raises(ValueError):
            cuda_runtime.linear(m, np.zeros((1, 32), np.float32))
    finally:
        m.close()
    with pytest.raises(RuntimeError, match="at most 49152 columns"):
        cuda_runtime.upload(np.zeros((1, 49168 // 2), np.uint8), np.zeros((1, 49168 // 16), np.uint8), 1.0)
    with pytest.raises(RuntimeError, match="invalid native NVFP4 matrix arguments"):
        cuda_runtime.upload(np.zeros((4, 4), np.uint8), np.zeros((4, 1), np.uint8), 0.0)
