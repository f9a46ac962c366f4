"""Masked temperature / top-p sampling on the GPU.

Mirrors the reference's seeded sampling surface (onyx_cuda/src/onyx_cuda/selection.py
``TemperatureTopPSelection``; torch_selection.py ``create_cuda_sampler``, whose session is
called with one logits row and returns an int) and adds a batched, masked form,
:func:`masked_sample`. The distribution and the kept top-p set are the reference's
(``_filtered_reference_weights``, float64). The random stream is this library's own:
Philox4x32-10 keyed by the seed, one counter per (call, row), so a session replays
identically from its seed (the reference's CUDA sampler uses torch's generator, whose
sequence no other implementation reproduces).
"""

from __future__ import annotations

import math
import threading
from dataclasses import dataclass
from typing import Any

import torch

from . import _lib
from . import masked_selection as _ms
from .torch_backend import TorchBackendExecutionError, TorchBackendInvariantError

__all__ = ["TemperatureTopPSelection", "MAX_SAMPLING_SEED", "masked_sample", "create_cuda_sampler"]

MAX_SAMPLING_SEED = (1 << 63) - 1


def _validate_parameter(value: float, *, label: str, minimum_exclusive: float,
                        maximum_inclusive: float | None) -> None:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{label} must be a real number")
    numeric = float(value)
    if not math.isfinite(numeric):
        raise ValueError(f"{label} must be finite")
    if numeric <= minimum_exclusive:
        raise ValueError(f"{label} must be greater than {minimum_exclusive}")
    if maximum_inclusive is not None and numeric > maximum_inclusive:
        raise ValueError(f"{label} must be at most {maximum_inclusive}")


@dataclass(frozen=True, slots=True)
class TemperatureTopPSelection:
    """Seeded temperature and nucleus-sampling policy (same fields and checks as the
    reference's): temperature finite and positive, top_p within (0, 1], seed a
    non-negative 63-bit integer."""

    temperature: float
    top_p: float
    seed: int

    def __post_init__(self) -> None:
        _validate_parameter(self.temperature, label="temperature", minimum_exclusive=0.0,
                            maximum_inclusive=None)
        _validate_parameter(self.top_p, label="top_p", minimum_exclusive=0.0,
                            maximum_inclusive=1.0)
        if isinstance(self.seed, bool) or not isinstance(self.seed, int):
            raise TypeError("seed must be an integer")
        if self.seed < 0 or self.seed > MAX_SAMPLING_SEED:
            raise ValueError(f"seed must be within [0, {MAX_SAMPLING_SEED}]")


def masked_sample(logits: torch.Tensor, bitmask: torch.Tensor | None = None, *,
                  temperature: float, top_p: float, seed: int,
                  call: int = 0) -> _ms.MaskedArgmaxResult:
    """One draw per row: ``token_ids`` int32[B] (-1 with a status) and ``status`` int32[B]
    (EMPTY_MASK, ALL_NEG_INF, NAN_IN_SUPPORT). Row r of call c draws Philox(seed; c, r):
    the same arguments give the same tokens."""
    policy = TemperatureTopPSelection(temperature, top_p, seed)
    if isinstance(call, bool) or not isinstance(call, int) or not 0 <= call < 1 << 64:
        raise ValueError("call must be an integer in [0, 2^64)")
    x = _ms._logits_2d(logits, "logits")
    rows, vocab = x.shape
    if x.dtype == torch.float64:
        raise TypeError("masked sampling supports float32/float16/bfloat16 logits")
    m = None if bitmask is None else _ms._mask_2d(bitmask, rows, vocab, "bitmask")
    device = x.device if m is None else _ms._same_device(x, m)
    idx = torch.empty(rows, dtype=torch.int32, device=device)
    status = torch.empty(rows, dtype=torch.int32, device=device)
    if rows == 0:
        return _ms.MaskedArgmaxResult(idx, status)
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        _lib.check(
            "onyx_masked_sample",
            lib.onyx_masked_sample(
                x.data_ptr(), _ms.dtype_code(x.dtype), rows, vocab,
                x.stride(0) if rows > 1 else vocab, None if m is None else m.data_ptr(),
                0 if m is None else m.stride(0), float(policy.temperature),
                float(policy.top_p), int(policy.seed), int(call), idx.data_ptr(),
                status.data_ptr(), stream.cuda_stream,
            ),
        )
    return _ms.MaskedArgmaxResult(idx, status)


class _CudaSamplingSession:
    """One seeded session: each call draws the next counter value."""

    def __init__(self, policy: TemperatureTopPSelection, device: torch.device) -> None:
        self._policy = policy
        self._device = device
        self._calls = 0
        self._lock = threading.Lock()

    def __call__(self, logits: Any) -> int:
        shape = tuple(getattr(logits, "shape", ()))
        if len(shape) != 1 or shape[0] <= 0:
            raise TorchBackendInvariantError(
                "CUDA sampling requires one nonempty logits row; "
                f"received shape {shape}")
        if not bool(getattr(logits, "is_cuda", False)):
            raise TorchBackendInvariantError("CUDA sampling received a non-CUDA tensor")
        if str(logits.device) != str(self._device):
            raise TorchBackendInvariantError(
                f"CUDA sampling received logits on {logits.device}; expected {self._device}")
        if not logits.is_floating_point():
            raise TorchBackendInvariantError("CUDA sampling logits must use a floating-point dtype")
        row = logits if logits.dtype != torch.float64 else logits.to(torch.float32)
        with self._lock:
            call = self._calls
            self._calls += 1
        try:
            r = masked_sample(row[None], temperature=self._policy.temperature,
                              top_p=self._policy.top_p, seed=self._policy.seed, call=call)
            both = torch.stack((r.token_ids, r.status)).cpu()
        except (TorchBackendInvariantError, TypeError, ValueError):
            raise
        except Exception as exc:
            raise TorchBackendExecutionError(f"CUDA sampling failed: {exc}") from exc
        selected, status = int(both[0, 0]), int(both[1, 0])
        if status & _ms.STATUS_NAN_IN_SUPPORT:
            raise TorchBackendInvariantError("CUDA sampling logits cannot contain NaN")
        if status & (_ms.STATUS_ALL_NEG_INF | _ms.STATUS_EMPTY_MASK):
            raise TorchBackendInvariantError("CUDA sampling logits cannot all be -inf")
        if selected < 0 or selected >= shape[0]:
            raise TorchBackendInvariantError(
                f"CUDA sampling returned token ID {selected} outside logits range [0, {shape[0]})")
        return selected


def create_cuda_sampler(policy: TemperatureTopPSelection, *,
                        device_index: int = 0) -> _CudaSamplingSession:
    """A private seeded sampler: calls return one token id per logits row (same policy,
    same sequence). Mirrors the reference's create_cuda_sampler."""
    if not isinstance(policy, TemperatureTopPSelection):
        raise TypeError("policy must be a TemperatureTopPSelection")
    if isinstance(device_index, bool) or not isinstance(device_index, int):
        raise TypeError("device_index must be an integer")
    if device_index < 0:
        raise ValueError("device_index cannot be negative")
    return _CudaSamplingSession(policy, torch.device(f"cuda:{device_index}"))
