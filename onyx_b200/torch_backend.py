"""Drop-in ``select_cuda_argmax`` backed by the sm_100a selection kernel.

Mirrors onyx_cuda/src/onyx_cuda/torch_backend.py:970-1007: one non-empty CUDA row, NaN
rejected, first (lowest-index) maximum returned as a Python int. The reference runs two
reductions and two device->host syncs (``isnan().any().item()`` then
``argmax().item()``); here one kernel produces the index and the NaN status together and
one 8-byte read brings both back.
"""

from __future__ import annotations

import torch

from . import masked_selection as _ms

__all__ = [
    "TorchBackendError",
    "TorchBackendExecutionError",
    "TorchBackendInvariantError",
    "select_cuda_argmax",
    "select_masked_cuda_argmax",
]


class TorchBackendError(RuntimeError):
    """Base error raised by the CUDA greedy selector (reference: BackendError subclass)."""


class TorchBackendExecutionError(TorchBackendError):
    """Raised when the CUDA selection kernel cannot execute."""


class TorchBackendInvariantError(TorchBackendError):
    """Raised when logits violate the selector contract (shape, device, NaN)."""


def _validate_row(logits) -> int:
    try:
        shape = tuple(logits.shape)
    except Exception as exc:
        raise TorchBackendInvariantError(f"CUDA logits shape could not be read: {exc}") from exc
    if len(shape) != 1 or not shape or shape[0] <= 0:
        raise TorchBackendInvariantError(
            f"CUDA greedy selector requires one nonempty logits row; received shape {shape}"
        )
    if not bool(getattr(logits, "is_cuda", False)):
        raise TorchBackendInvariantError("CUDA greedy selector received a non-CUDA tensor")
    device = getattr(logits, "device", None)
    device_text = str(device)
    if device is None or not (device_text == "cuda" or device_text.startswith("cuda:")):
        raise TorchBackendInvariantError(
            f"CUDA greedy selector received logits on {device}; expected a CUDA device"
        )
    return shape[0]


def _read_selection(result: _ms.MaskedArgmaxResult, vocab: int, *, masked: bool) -> int:
    try:
        both = torch.stack((result.token_ids, result.status)).cpu()
    except Exception as exc:
        raise TorchBackendExecutionError(f"CUDA argmax failed: {exc}") from exc
    selected, status = int(both[0, 0]), int(both[1, 0])
    if status & _ms.STATUS_WAIT_TIMEOUT:
        raise TorchBackendExecutionError("CUDA argmax failed: a bounded in-kernel wait gave up")
    if status & _ms.STATUS_NAN_IN_SUPPORT:
        raise TorchBackendInvariantError("CUDA logits cannot contain NaN")
    if masked and status & _ms.STATUS_EMPTY_MASK:
        raise TorchBackendInvariantError("CUDA greedy selector received an empty token mask")
    if masked and status & _ms.STATUS_ALL_NEG_INF:
        raise TorchBackendInvariantError("valid token IDs have no logit support above -inf")
    if selected < 0 or selected >= vocab:
        raise TorchBackendInvariantError(
            f"CUDA argmax returned token ID {selected} outside logits range [0, {vocab})"
        )
    return selected


def select_cuda_argmax(logits) -> int:
    """Select the first maximum on CUDA without transferring vocabulary logits to CPU."""
    vocab = _validate_row(logits)
    try:
        dtype_ok = logits.dtype in (torch.float32, torch.float16, torch.bfloat16, torch.float64)
    except Exception as exc:
        raise TorchBackendInvariantError(f"CUDA logits dtype could not be read: {exc}") from exc
    if not dtype_ok:
        raise TorchBackendInvariantError(f"CUDA greedy selector does not support {logits.dtype}")
    try:
        result = _ms.masked_argmax(logits, None)
    except Exception as exc:
        raise TorchBackendExecutionError(f"CUDA argmax failed: {exc}") from exc
    return _read_selection(result, vocab, masked=False)


def select_masked_cuda_argmax(logits, bitmask) -> int:
    """``select_cuda_argmax(mask.apply(logits, ids))`` in one pass, given the packed mask."""
    vocab = _validate_row(logits)
    try:
        result = _ms.masked_argmax(logits, bitmask)
    except Exception as exc:
        raise TorchBackendExecutionError(f"CUDA masked argmax failed: {exc}") from exc
    return _read_selection(result, vocab, masked=True)
