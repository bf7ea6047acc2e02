"""``nvfp4_moe::forward`` torch custom op over resident banks.

Banks are registered under an integer id (``register_bank``); the op takes
BF16 [tokens, hidden] CUDA tensors and returns the layer output with the
residual added. It launches on torch's current stream through
``nvfp4_moe_bank_forward_ptr_bf16``.
"""

from __future__ import annotations

import threading

import torch

from .runtime import MoeBank

_banks: dict[int, MoeBank] = {}
_lock = threading.Lock()


def register_bank(bank: MoeBank) -> int:
    with _lock:
        bank_id = len(_banks)
        _banks[bank_id] = bank
        return bank_id


@torch.library.custom_op("nvfp4_moe::forward", mutates_args=())
def forward(bank_id: int, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    bank = _banks[bank_id]
    return bank.forward(x, residual=residual)


@forward.register_fake
def _(bank_id: int, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    return torch.empty_like(x)
