"""The vLLM plugin hook: x2-nvfp4-lab_b200/pyproject.toml declares
``vllm_nvfp4_cuda:register`` in the ``vllm.general_plugins`` group, as the
lab declares ``vllm_nvfp4_opencl:register``
(vllm_nvfp4_opencl/pyproject.toml:12-13).

The package is installed (offline, no dependencies) into a temporary
directory, and a fresh interpreter with only that directory added runs
vLLM's own plugin loader: the entry point must be discovered through
``importlib.metadata`` and its call must register the CUDA linear provider.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "x2-nvfp4-lab_b200"

_CHILD = r"""
import importlib.metadata as md
eps = [ep for ep in md.entry_points(group="vllm.general_plugins") if ep.name == "nvidia_nvfp4_cuda"]
assert len(eps) == 1, eps
assert eps[0].value == "vllm_nvfp4_cuda:register", eps[0].value
import vllm_nvfp4_cuda
assert vllm_nvfp4_cuda.__file__.startswith(SITE), vllm_nvfp4_cuda.__file__
from vllm.plugins import load_general_plugins
load_general_plugins()
from vllm.model_executor.kernels import linear as kl
from vllm.platforms import PlatformEnum
from vllm_nvfp4_cuda.linear import CudaNvFp4LinearKernel
assert kl._POSSIBLE_NVFP4_KERNELS[PlatformEnum.CUDA].count(CudaNvFp4LinearKernel) == 1
print("PLUGIN_OK")
"""


def test_general_plugins_entry_point_registers_provider(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    shutil.copy(PKG / "pyproject.toml", src / "pyproject.toml")
    shutil.copytree(PKG / "vllm_nvfp4_cuda", src / "vllm_nvfp4_cuda",
                    ignore=shutil.ignore_patterns("__pycache__", "*.so"))
    site = tmp_path / "site"
    subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                    "--quiet", "--target", str(site), str(src)], check=True, capture_output=True, timeout=300)
    code = f"import sys; sys.path.insert(0, {str(site)!r}); SITE = {str(site)!r}\n" + _CHILD
    proc = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                          cwd=str(tmp_path), env={"PATH": "/usr/bin:/bin", "VLLM_LOGGING_LEVEL": "ERROR",
                                                  "HOME": str(tmp_path)})
    assert proc.returncode == 0 and "PLUGIN_OK" in proc.stdout, proc.stdout[-2000:] + proc.stderr[-4000:]
