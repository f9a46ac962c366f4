"""Drop-in CUDA grammar-logit mask for B200, behind the reference's mask boundary.

Same factory, class surface, argument checks and exception hierarchy as
onyx_cuda/src/onyx_cuda/torch_grammar_mask.py (``create_cuda_grammar_logit_mask`` :311,
``TorchCUDAGrammarLogitMask.apply`` :69-86, ``apply_with_timing`` :88-130, errors :18-35),
so ``GrammarLogitMask`` callers (constrained_generation.py:89-115, :295-315;
grammar_selection.py:129) run unchanged.

What differs is the transport and the device work. The reference copies the valid ids to
the GPU as ``int64`` (8 bytes per valid id) and runs ``index_select`` + ``full_like`` +
``index_copy_`` + ``isneginf().all()``; this mask packs the ids into the bitmask layout on
the host (V/8 bytes, pinned), copies it asynchronously, and one sm_100a kernel writes the
masked row and the support check together. The support check still ends in one small
device->host read, as the reference's ``.item()`` does, because ``apply`` must raise
synchronously on an all ``-inf`` support.
"""

from __future__ import annotations

import importlib
import math
import threading
import time
from collections.abc import Callable
from typing import Any

import numpy as np

from . import bitmask as _bitmask

__all__ = [
    "TorchGrammarMaskError",
    "TorchGrammarMaskImportError",
    "TorchGrammarMaskUnavailableError",
    "TorchGrammarMaskInvariantError",
    "TorchGrammarMaskExecutionError",
    "TorchCUDAGrammarLogitMask",
    "B200GrammarLogitMask",
    "create_cuda_grammar_logit_mask",
]

_BITMASK_TRANSPORT = "packed_bitmask"


class TorchGrammarMaskError(RuntimeError):
    """Base error raised by the PyTorch CUDA grammar-logit mask boundary."""


class TorchGrammarMaskImportError(TorchGrammarMaskError):
    """Raised when PyTorch cannot be imported for explicit mask creation."""


class TorchGrammarMaskUnavailableError(TorchGrammarMaskError):
    """Raised when the requested CUDA mask device is unavailable."""


class TorchGrammarMaskInvariantError(TorchGrammarMaskError):
    """Raised when logits, valid IDs, or mask results violate the boundary contract."""


class TorchGrammarMaskExecutionError(TorchGrammarMaskError):
    """Raised when a PyTorch or CUDA mask operation cannot execute."""


class B200GrammarLogitMask:
    """Apply one valid-token set to a CUDA logits row with the sm_100a mask kernel."""

    def __init__(
        self,
        *,
        torch_module: Any,
        vocab_size: int,
        device_index: int,
        device: Any,
        clock: Callable[[], float],
    ) -> None:
        self._torch = torch_module
        self._vocab_size = vocab_size
        self._device_index = device_index
        self._device = device
        self._transport_name = _BITMASK_TRANSPORT
        self._clock = clock
        self._words = _bitmask.words_for(vocab_size)
        self._lock = threading.Lock()
        self._host_words: Any = None  # pinned staging buffer, reused
        self._copy_done: Any = None  # event recorded after the last copy out of it

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    @property
    def device_index(self) -> int:
        return self._device_index

    @property
    def transport_name(self) -> str:
        return self._transport_name

    # -- reference surface ---------------------------------------------------------------
    def apply(self, logits: Any, valid_token_ids: tuple[int, ...], /) -> Any:
        """Return a new row preserving only logits named by a valid-ID tuple."""
        _validate_valid_token_ids(valid_token_ids, self._vocab_size)
        self._validate_logits(logits)
        words = self._materialize_device_words(valid_token_ids)
        return self._apply_device_words(logits, words)

    def apply_with_timing(
        self,
        logits: Any,
        valid_token_ids: tuple[int, ...],
        timing_session: Any,
        /,
    ) -> Any:
        """Apply the mask and record synchronized transfer/application wall times."""
        if not callable(getattr(timing_session, "record_mask_timing", None)):
            raise TypeError("timing_session must be a GrammarTimingSession")
        _validate_valid_token_ids(valid_token_ids, self._vocab_size)
        self._validate_logits(logits)
        self._synchronize("before valid-index transfer")
        transfer_start = self._read_clock()
        words = self._materialize_device_words(valid_token_ids)
        self._synchronize("after valid-index transfer")
        transfer_end = self._read_clock()
        transfer_time = self._elapsed(transfer_start, transfer_end, label="valid-index transfer")
        application_start = self._read_clock()
        result = self._apply_device_words(logits, words)
        self._synchronize("after mask application")
        application_end = self._read_clock()
        application_time = self._elapsed(
            application_start, application_end, label="mask application"
        )
        timing_session.record_mask_timing(transfer_time, application_time)
        return result

    # -- bitmask surface (no host packing) -----------------------------------------------
    def apply_bitmask(self, logits: Any, bitmask: Any, /) -> Any:
        """Like :meth:`apply` with the valid set already packed on the device."""
        self._validate_logits(logits)
        if not getattr(bitmask, "is_cuda", False) or str(bitmask.device) != str(self._device):
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar bitmask must live on {self._device}"
            )
        return self._apply_device_words(logits, bitmask)

    # -- internals -------------------------------------------------------------------------
    def _materialize_device_words(self, valid_token_ids: tuple[int, ...]) -> Any:
        torch = self._torch
        try:
            with self._lock:
                if self._host_words is None:
                    self._host_words = torch.zeros(
                        self._words, dtype=torch.int32, pin_memory=True
                    )
                host = self._host_words
                if self._copy_done is not None:
                    self._copy_done.synchronize()  # the previous copy has left the buffer
                _bitmask.pack_ids(
                    np.asarray(valid_token_ids, dtype=np.int64),
                    self._vocab_size,
                    out=host.numpy().view(np.uint32),
                )
                device_words = host.to(device=self._device, non_blocking=True)
                if self._copy_done is None:
                    self._copy_done = torch.cuda.Event()
                self._copy_done.record(torch.cuda.current_stream(self._device))
            return device_words
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(
                f"CUDA grammar-logit mask preparation failed: {exc}"
            ) from exc

    def _apply_device_words(self, logits: Any, words: Any) -> Any:
        from . import masked_selection as _ms

        try:
            result, status = _ms.mask_apply(logits, words)
            status_value = int(status[0].item())
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(
                f"CUDA grammar-logit mask application failed: {exc}"
            ) from exc
        if result is logits:
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar mask result must not alias the input tensor"
            )
        if status_value & _ms.STATUS_EMPTY_MASK:
            raise TorchGrammarMaskInvariantError("valid_token_ids cannot be empty")
        if status_value & _ms.STATUS_ALL_NEG_INF:
            raise TorchGrammarMaskInvariantError("valid token IDs have no logit support above -inf")
        return result

    def _synchronize(self, boundary: str) -> None:
        try:
            self._torch.cuda.synchronize(self._device)
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(
                f"CUDA grammar-logit mask synchronization failed {boundary}: {exc}"
            ) from exc

    def _read_clock(self) -> float:
        try:
            value = self._clock()
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(
                f"CUDA grammar-logit timing clock failed: {exc}"
            ) from exc
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar-logit timing clock must return a real number"
            )
        numeric = float(value)
        if not math.isfinite(numeric):
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar-logit timing clock must return a finite value"
            )
        return numeric

    @staticmethod
    def _elapsed(start: float, end: float, *, label: str) -> float:
        duration = end - start
        if not math.isfinite(duration):
            raise TorchGrammarMaskInvariantError(f"{label} duration must be finite")
        if duration < 0.0:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar-logit timing clock moved backwards during {label}"
            )
        return duration

    def _validate_logits(self, logits: Any) -> None:
        try:
            shape = tuple(logits.shape)
        except Exception as exc:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar logits shape could not be read: {exc}"
            ) from exc
        if shape != (self._vocab_size,):
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar mask requires one logits row with configured vocabulary shape "
                f"({self._vocab_size},); received {shape}"
            )
        try:
            is_cuda = bool(logits.is_cuda)
            device_text = str(logits.device)
            expected_device_text = str(self._device)
        except Exception as exc:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar logits device could not be read: {exc}"
            ) from exc
        if not is_cuda:
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar mask received a non-CUDA logits tensor"
            )
        if device_text != expected_device_text:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar mask received logits on {device_text}; expected {expected_device_text}"
            )
        try:
            is_floating_point = bool(logits.is_floating_point())
            dtype = logits.dtype
        except Exception as exc:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar logits dtype could not be validated: {exc}"
            ) from exc
        torch = self._torch
        if not is_floating_point or dtype not in (
            torch.float16, torch.bfloat16, torch.float32, torch.float64
        ):
            raise TorchGrammarMaskInvariantError(
                "CUDA grammar logits must use a real floating-point dtype"
            )


# the reference's class name, for callers that construct or isinstance-check it
TorchCUDAGrammarLogitMask = B200GrammarLogitMask


def create_cuda_grammar_logit_mask(
    vocab_size: int,
    *,
    device_index: int = 0,
    clock: Callable[[], float] = time.perf_counter,
) -> B200GrammarLogitMask:
    """Create a stateless mask on one CUDA device, importing PyTorch only now."""
    _validate_factory_inputs(vocab_size, device_index, clock)
    try:
        torch_module = importlib.import_module("torch")
    except (ImportError, OSError) as exc:
        raise TorchGrammarMaskImportError(
            f"PyTorch could not be imported for CUDA grammar masking: {exc}"
        ) from exc
    return _create_cuda_grammar_logit_mask(
        torch_module, vocab_size, device_index=device_index, clock=clock
    )


def _create_cuda_grammar_logit_mask(
    torch_module: Any,
    vocab_size: int,
    *,
    device_index: int,
    clock: Callable[[], float] = time.perf_counter,
) -> B200GrammarLogitMask:
    _validate_factory_inputs(vocab_size, device_index, clock)
    try:
        cuda = torch_module.cuda
        cuda_available = cuda.is_available()
        device_count = cuda.device_count() if cuda_available else 0
    except Exception as exc:
        raise TorchGrammarMaskExecutionError(
            f"CUDA grammar-mask availability check failed: {exc}"
        ) from exc
    if not isinstance(cuda_available, bool):
        raise TorchGrammarMaskInvariantError(
            "CUDA grammar-mask availability result must be a boolean"
        )
    if not cuda_available:
        raise TorchGrammarMaskUnavailableError("PyTorch reports that CUDA is unavailable")
    if isinstance(device_count, bool) or not isinstance(device_count, int):
        raise TorchGrammarMaskInvariantError("CUDA device count must be an integer")
    if device_count < 0:
        raise TorchGrammarMaskInvariantError("CUDA device count cannot be negative")
    if device_index >= device_count:
        raise TorchGrammarMaskUnavailableError(
            f"CUDA device index {device_index} is unavailable; detected {device_count} device(s)"
        )
    try:
        device = torch_module.device(f"cuda:{device_index}")
    except Exception as exc:
        raise TorchGrammarMaskExecutionError(
            f"CUDA grammar-mask device creation failed: {exc}"
        ) from exc
    return B200GrammarLogitMask(
        torch_module=torch_module,
        vocab_size=vocab_size,
        device_index=device_index,
        device=device,
        clock=clock,
    )


def _validate_factory_inputs(vocab_size: int, device_index: int, clock: Callable[[], float]) -> None:
    if isinstance(vocab_size, bool) or not isinstance(vocab_size, int):
        raise TypeError("vocab_size must be an integer")
    if vocab_size <= 0:
        raise ValueError("vocab_size must be greater than zero")
    if isinstance(device_index, bool) or not isinstance(device_index, int):
        raise TypeError("device_index must be an integer")
    if device_index < 0:
        raise ValueError("device_index cannot be negative")
    if not callable(clock):
        raise TypeError("clock must be callable")


def _validate_valid_token_ids(valid_token_ids: tuple[int, ...], vocab_size: int) -> None:
    if not isinstance(valid_token_ids, tuple):
        raise TorchGrammarMaskInvariantError("valid_token_ids must be a tuple")
    if not valid_token_ids:
        raise TorchGrammarMaskInvariantError("valid_token_ids cannot be empty")
    previous = -1
    for token_id in valid_token_ids:
        if isinstance(token_id, bool) or not isinstance(token_id, int):
            raise TorchGrammarMaskInvariantError(
                "valid_token_ids must contain only Python integers"
            )
        if token_id < 0 or token_id >= vocab_size:
            raise TorchGrammarMaskInvariantError(
                f"valid token ID {token_id} is outside vocabulary range [0, {vocab_size})"
            )
        if token_id <= previous:
            raise TorchGrammarMaskInvariantError(
                "valid_token_ids must be strictly increasing and unique"
            )
        previous = token_id
