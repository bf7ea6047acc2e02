"""The C-ABI library loads and exports every symbol include/*.h declares
(no compute call is made; these run without a GPU)."""

from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER_DIR = ROOT / "include"


def declared_symbols() -> list[str]:
    names = []
    for header in sorted(HEADER_DIR.glob("*.h")):
        text = header.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"NVFP4_API\s+[^;(]*?\b(nvfp4_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def library_path():
    sys_path_pkg = ROOT / "x2-nvfp4-lab_b200"
    lib = sys_path_pkg / "vllm_nvfp4_cuda" / "lib" / "libnvfp4_moe_cuda.so"
    if not lib.exists():
        subprocess.run(["python", str(sys_path_pkg / "build.py")], check=True)
    return lib


def test_header_declares_reference_hot_path():
    names = set(declared_symbols())
    for required in (
        "nvfp4_runtime_create", "nvfp4_runtime_destroy", "nvfp4_runtime_device_name", "nvfp4_last_error",
        "nvfp4_runtime_last_profile", "nvfp4_runtime_synchronize", "nvfp4_runtime_trace_set_enabled",
        "nvfp4_runtime_trace_set_scope", "nvfp4_runtime_trace_count", "nvfp4_runtime_trace_read",
        "nvfp4_buffer_create", "nvfp4_buffer_destroy", "nvfp4_buffer_upload", "nvfp4_buffer_download",
        "nvfp4_buffer_copy_enqueue", "nvfp4_add_device_enqueue_f32", "nvfp4_rmsnorm_device_enqueue_f32",
        "nvfp4_weighted_accumulate_device_enqueue_f32", "nvfp4_silu_mul_device_enqueue_f32",
        "nvfp4_bf16_gemv_device_enqueue", "nvfp4_moe_bank_create", "nvfp4_moe_bank_upload_projection",
        "nvfp4_moe_bank_decode_device_enqueue_f32", "nvfp4_moe_bank_destroy",
    ):
        assert required in names, required


def test_library_exports_every_declared_symbol(library_path):
    lib = C.CDLL(str(library_path))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_exports_nothing_else(library_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(library_path)], capture_output=True, text=True,
                         check=True).stdout
    exported = sorted({line.split()[-1] for line in out.splitlines() if line.strip()} - {"nvfp4_"})
    assert set(exported) == set(declared_symbols())


def test_python_layer_declares_every_symbol():
    import vllm_nvfp4_cuda.runtime as rt

    assert set(rt._SIGNATURES) == set(declared_symbols())


def test_runtime_create_reports_missing_device(library_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from vllm_nvfp4_cuda.runtime import Runtime

    with pytest.raises(RuntimeError, match=r"runtime_create failed \(2\)"):
        Runtime(library_path)


def test_provider_gate(monkeypatch):
    from vllm_nvfp4_cuda.runtime import provider_enabled

    monkeypatch.delenv("VLLM_NVFP4_CUDA", raising=False)
    ok, reason = provider_enabled()
    assert not ok and "VLLM_NVFP4_CUDA=1" in reason


def test_custom_op_fake_kernel():
    """register() defines torch.ops.nvfp4_moe.forward with a fake kernel, so
    model code that calls a bank can be traced (torch.compile, graph capture
    planning) without the library: under FakeTensorMode the op returns a
    tensor shaped like x."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    import vllm_nvfp4_cuda

    vllm_nvfp4_cuda.register()
    vllm_nvfp4_cuda.register()  # idempotent
    op = torch.ops.nvfp4_moe.forward
    with FakeTensorMode():
        x = torch.empty(3, 2048, dtype=torch.bfloat16)
        y = op(0, x, torch.empty_like(x))
        assert y.shape == x.shape and y.dtype == x.dtype
