"""Drop-in CUDA grammar-logit mask for B200, behind the reference's mask boundary.

The contract kept from onyx_cuda/src/onyx_cuda/torch_grammar_mask.py is the surface callers
depend on: the factory ``create_cuda_grammar_logit_mask(vocab_size, *, device_index=0,
clock=time.perf_counter)`` (:311), the class name ``TorchCUDAGrammarLogitMask`` with
``vocab_size``, ``device_index``, ``transport_name``, ``apply`` (:69-86) and
``apply_with_timing`` (:88-130), the exception types (:18-35) and the message fragments that
callers and the reference's tests match on. ``GrammarLogitMask`` callers
(constrained_generation.py:89-115, :295-315; grammar_selection.py:129) run unchanged.

Everything behind that surface is this package's own:

* validation is a list of rules per input, each a predicate with the exception it raises;
  valid-id tuples are checked with one vectorised pass instead of a loop per id;
* the valid ids travel as the packed bitmask (V/8 bytes in a reused pinned buffer, one
  asynchronous copy) instead of ``int64`` ids (8 bytes per valid id);
* one sm_100a kernel writes the masked row and its support check together, instead of
  ``index_select`` + ``full_like`` + ``index_copy_`` + ``isneginf().all()``. The support
  check still ends in one small device->host read, as the reference's ``.item()`` does,
  because ``apply`` must raise synchronously on an all ``-inf`` support.
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
_FLOAT_DTYPE_NAMES = ("float16", "bfloat16", "float32", "float64")


class TorchGrammarMaskError(RuntimeError):
    """Common base of every error this mask raises."""


class TorchGrammarMaskImportError(TorchGrammarMaskError):
    """PyTorch itself failed to import when a mask was requested."""


class TorchGrammarMaskUnavailableError(TorchGrammarMaskError):
    """No usable CUDA device answers to the requested index."""


class TorchGrammarMaskInvariantError(TorchGrammarMaskError):
    """An input (logits row, valid ids, clock reading) or a result breaks the contract."""


class TorchGrammarMaskExecutionError(TorchGrammarMaskError):
    """A device operation (query, copy, kernel, synchronisation) raised."""


# ---------------------------------------------------------------------------------------
# rules: each is (predicate that holds for a good value, exception type, message)
# ---------------------------------------------------------------------------------------
def _is_int(v: object) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


_FACTORY_RULES: tuple[tuple[str, Callable[[object], bool], type[Exception], str], ...] = (
    ("vocab_size", _is_int, TypeError, "vocab_size must be an integer"),
    ("vocab_size", lambda v: v > 0, ValueError, "vocab_size must be greater than zero"),
    ("device_index", _is_int, TypeError, "device_index must be an integer"),
    ("device_index", lambda v: v >= 0, ValueError, "device_index cannot be negative"),
    ("clock", callable, TypeError, "clock must be callable"),
)


def _check_factory_arguments(**values: object) -> None:
    for name, holds, error, message in _FACTORY_RULES:
        if not holds(values[name]):
            raise error(message)


def _validate_factory_inputs(vocab_size: int, device_index: int, clock: Callable[[], float]) -> None:
    _check_factory_arguments(vocab_size=vocab_size, device_index=device_index, clock=clock)


def _valid_ids_array(valid_token_ids: object, vocab_size: int) -> np.ndarray:
    """The valid ids as int64 after the boundary's rules: a non-empty tuple of Python
    integers (bool excluded), each in [0, vocab_size), strictly increasing."""
    bad = TorchGrammarMaskInvariantError
    if type(valid_token_ids) is not tuple:
        raise bad("valid_token_ids must be a tuple")
    if not valid_token_ids:
        raise bad("valid_token_ids cannot be empty")
    if not set(map(type, valid_token_ids)) <= {int}:
        raise bad("valid_token_ids must contain only Python integers")
    try:
        ids = np.asarray(valid_token_ids, dtype=np.int64)
    except OverflowError:
        ids = None
    if ids is None or int(ids.min()) < 0 or int(ids.max()) >= vocab_size:
        out = next(t for t in valid_token_ids if t < 0 or t >= vocab_size)
        raise bad(f"valid token ID {out} is outside vocabulary range [0, {vocab_size})")
    if ids.size > 1 and not bool(np.all(ids[1:] > ids[:-1])):
        raise bad("valid_token_ids must be strictly increasing and unique")
    return ids


def _validate_valid_token_ids(valid_token_ids: tuple[int, ...], vocab_size: int) -> None:
    _valid_ids_array(valid_token_ids, vocab_size)


def _read_or_invariant(read: Callable[[], Any], what: str) -> Any:
    """Reads tensor metadata; a failure becomes the boundary's invariant error."""
    try:
        return read()
    except Exception as exc:
        raise TorchGrammarMaskInvariantError(f"CUDA grammar logits {what} could not be read: {exc}") from exc


class _Stopwatch:
    """Wall-clock spans from the caller's clock, which must give finite, non-decreasing
    real numbers; a clock that raises is an execution failure."""

    def __init__(self, clock: Callable[[], float]) -> None:
        self._clock = clock

    def now(self) -> float:
        try:
            value = self._clock()
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(f"CUDA grammar-logit timing clock failed: {exc}") from exc
        if not isinstance(value, (int, float)) or isinstance(value, bool):
            raise TorchGrammarMaskInvariantError("CUDA grammar-logit timing clock must return a real number")
        if not math.isfinite(value):
            raise TorchGrammarMaskInvariantError("CUDA grammar-logit timing clock must return a finite value")
        return float(value)

    @staticmethod
    def span(start: float, end: float, label: str) -> float:
        seconds = end - start
        if not math.isfinite(seconds):
            raise TorchGrammarMaskInvariantError(f"{label} duration must be finite")
        if seconds < 0.0:
            raise TorchGrammarMaskInvariantError(f"CUDA grammar-logit timing clock moved backwards during {label}")
        return seconds


# ---------------------------------------------------------------------------------------
class B200GrammarLogitMask:
    """One valid-token set applied to one CUDA logits row by the sm_100a mask kernel.

    Stateless between calls apart from a reused pinned staging buffer for the packed
    valid set; no reference to an input or an output is kept."""

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
        self._device_text = str(device)
        self._stopwatch = _Stopwatch(clock)
        self._words = _bitmask.words_for(vocab_size)
        self._staging_lock = threading.Lock()
        self._staging: Any = None  # pinned int32[words], reused across calls
        self._staging_free: Any = None  # event: the last copy out of the staging buffer ended

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    @property
    def device_index(self) -> int:
        return self._device_index

    @property
    def transport_name(self) -> str:
        return _BITMASK_TRANSPORT

    # -- reference surface ---------------------------------------------------------------
    def apply(self, logits: Any, valid_token_ids: tuple[int, ...], /) -> Any:
        """A new row: the logits at the valid ids bit for bit, ``-inf`` everywhere else."""
        ids = _valid_ids_array(valid_token_ids, self._vocab_size)
        self._check_row(logits)
        return self._masked_row(logits, self._upload(ids))

    def apply_with_timing(self, logits: Any, valid_token_ids: tuple[int, ...],
                          timing_session: Any, /) -> Any:
        """``apply``, recording the (transfer, application) seconds with the session; the
        device is synchronised around each part so the spans are wall-clock work."""
        if not callable(getattr(timing_session, "record_mask_timing", None)):
            raise TypeError("timing_session must be a GrammarTimingSession")
        ids = _valid_ids_array(valid_token_ids, self._vocab_size)
        self._check_row(logits)
        watch = self._stopwatch
        self._sync("before valid-index transfer")
        t0 = watch.now()
        words = self._upload(ids)
        self._sync("after valid-index transfer")
        t1 = watch.now()
        transfer = watch.span(t0, t1, "valid-index transfer")
        t2 = watch.now()
        row = self._masked_row(logits, words)
        self._sync("after mask application")
        t3 = watch.now()
        timing_session.record_mask_timing(transfer, watch.span(t2, t3, "mask application"))
        return row

    # -- bitmask surface (no host packing) -----------------------------------------------
    def apply_bitmask(self, logits: Any, bitmask: Any, /) -> Any:
        """Like :meth:`apply` with the valid set already packed on the device."""
        self._check_row(logits)
        if not getattr(bitmask, "is_cuda", False) or str(bitmask.device) != self._device_text:
            raise TorchGrammarMaskInvariantError(f"CUDA grammar bitmask must live on {self._device}")
        return self._masked_row(logits, bitmask)

    # -- internals -------------------------------------------------------------------------
    def _check_row(self, logits: Any) -> None:
        shape = tuple(_read_or_invariant(lambda: logits.shape, "shape"))
        if shape != (self._vocab_size,):
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar mask requires one logits row with configured vocabulary shape "
                f"({self._vocab_size},); received {shape}")
        on_cuda = bool(_read_or_invariant(lambda: logits.is_cuda, "device"))
        where = _read_or_invariant(lambda: str(logits.device), "device")
        if not on_cuda:
            raise TorchGrammarMaskInvariantError("CUDA grammar mask received a non-CUDA logits tensor")
        if where != self._device_text:
            raise TorchGrammarMaskInvariantError(
                f"CUDA grammar mask received logits on {where}; expected {self._device_text}")
        floating = bool(_read_or_invariant(lambda: logits.is_floating_point(), "dtype"))
        dtype_name = str(_read_or_invariant(lambda: logits.dtype, "dtype")).rpartition(".")[2]
        if not floating or dtype_name not in _FLOAT_DTYPE_NAMES:
            raise TorchGrammarMaskInvariantError("CUDA grammar logits must use a real floating-point dtype")

    def _upload(self, ids: np.ndarray) -> Any:
        """The packed valid set on the device: packed into the pinned staging buffer once its
        previous copy has left, then one asynchronous copy on the current stream."""
        torch = self._torch
        try:
            with self._staging_lock:
                if self._staging is None:
                    self._staging = torch.zeros(self._words, dtype=torch.int32, pin_memory=True)
                    self._staging_free = torch.cuda.Event()
                else:
                    self._staging_free.synchronize()
                _bitmask.pack_ids(ids, self._vocab_size, out=self._staging.numpy().view(np.uint32))
                words = self._staging.to(device=self._device, non_blocking=True)
                self._staging_free.record(torch.cuda.current_stream(self._device))
            return words
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(f"CUDA grammar-logit mask preparation failed: {exc}") from exc

    def _masked_row(self, logits: Any, words: Any) -> Any:
        from . import masked_selection as _ms

        try:
            row, status = _ms.mask_apply(logits, words)
            bits = int(status[0].item())
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(f"CUDA grammar-logit mask application failed: {exc}") from exc
        if row is logits:
            raise TorchGrammarMaskInvariantError("CUDA grammar mask result must not alias the input tensor")
        if bits & _ms.STATUS_EMPTY_MASK:
            raise TorchGrammarMaskInvariantError("valid_token_ids cannot be empty")
        if bits & _ms.STATUS_ALL_NEG_INF:
            raise TorchGrammarMaskInvariantError("valid token IDs have no logit support above -inf")
        return row

    def _sync(self, when: str) -> None:
        try:
            self._torch.cuda.synchronize(self._device)
        except Exception as exc:
            raise TorchGrammarMaskExecutionError(
                f"CUDA grammar-logit mask synchronization failed {when}: {exc}") from exc


# the reference's class name, for callers that construct or isinstance-check it
TorchCUDAGrammarLogitMask = B200GrammarLogitMask


def create_cuda_grammar_logit_mask(
    vocab_size: int,
    *,
    device_index: int = 0,
    clock: Callable[[], float] = time.perf_counter,
) -> B200GrammarLogitMask:
    """A mask for ``vocab_size`` tokens on CUDA device ``device_index``; PyTorch is imported
    here, at creation, not at package import."""
    _check_factory_arguments(vocab_size=vocab_size, device_index=device_index, clock=clock)
    try:
        torch_module = importlib.import_module("torch")
    except (ImportError, OSError) as exc:
        raise TorchGrammarMaskImportError(f"PyTorch could not be imported for CUDA grammar masking: {exc}") from exc
    return _create_cuda_grammar_logit_mask(torch_module, vocab_size, device_index=device_index, clock=clock)


def _create_cuda_grammar_logit_mask(
    torch_module: Any,
    vocab_size: int,
    *,
    device_index: int,
    clock: Callable[[], float] = time.perf_counter,
) -> B200GrammarLogitMask:
    """The factory with PyTorch passed in (the seam tests use for a fake module)."""
    _check_factory_arguments(vocab_size=vocab_size, device_index=device_index, clock=clock)
    try:
        available = torch_module.cuda.is_available()
        count = torch_module.cuda.device_count() if available else 0
    except Exception as exc:
        raise TorchGrammarMaskExecutionError(f"CUDA grammar-mask availability failed: {exc}") from exc
    if type(available) is not bool:
        raise TorchGrammarMaskInvariantError("CUDA grammar-mask availability result must be a boolean")
    if not available:
        raise TorchGrammarMaskUnavailableError("CUDA unavailable: PyTorch reports no CUDA support")
    if not _is_int(count):
        raise TorchGrammarMaskInvariantError("CUDA device count must be an integer")
    if count < 0:
        raise TorchGrammarMaskInvariantError("CUDA device count cannot be negative")
    if device_index >= count:
        raise TorchGrammarMaskUnavailableError(
            f"CUDA device index {device_index} is unavailable; detected {count} device(s)")
    try:
        device = torch_module.device(f"cuda:{device_index}")
    except Exception as exc:
        raise TorchGrammarMaskExecutionError(f"CUDA grammar-mask device failed: {exc}") from exc
    return B200GrammarLogitMask(torch_module=torch_module, vocab_size=vocab_size,
                                device_index=device_index, device=device, clock=clock)
