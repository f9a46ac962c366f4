"""ctypes binding of ``libonyx_b200.so`` (C ABI declared in ``include/onyx_b200.h``).

The CUDA library is the only compute path of this package: there is no CPU or PyTorch
fallback. If the shared object is missing or cannot be loaded, every entry point raises
:class:`OnyxLibraryUnavailableError`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libonyx_b200.so"

ABI_VERSION = 1

DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_F64 = 0, 1, 2, 3

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_DTYPE = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_SCRATCH_LIMIT = 5
NOALLOC_SCRATCH_BYTES = 1 << 20

OPTION_CLUSTER = 0
OPTION_PDL = 1
OPTION_SAMPLE_FORM = 2
OPTION_TEST_WITHHELD_KEY_BYTES = 3

STATUS_EMPTY_MASK = 1
STATUS_ALL_NEG_INF = 2
STATUS_NAN_IN_SUPPORT = 4
STATUS_BAD_STATE = 8
STATUS_WAIT_TIMEOUT = 16

# every symbol include/onyx_b200.h declares, with its ctypes signature
_i64, _i32, _vp, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
SIGNATURES: dict[str, tuple[object, list]] = {
    "onyx_abi_version": (_i32, []),
    "onyx_error_string": (ctypes.c_char_p, [_i32]),
    "onyx_last_cuda_error": (_i32, []),
    "onyx_set_option": (_i32, [_i32, _i64]),
    "onyx_get_option": (_i64, [_i32]),
    "onyx_masked_argmax_workspace_size": (_sz, [_i64, _i64, _i32]),
    "onyx_masked_argmax": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _sz, _vp]),
    "onyx_gather_masked_argmax": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "onyx_spec_verify_workspace_size": (_sz, [_i64, _i64, _i64, _i32]),
    "onyx_spec_verify": (
        _i32,
        [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i32, _vp, _vp,
         _vp, _vp, _sz, _vp]),
    "onyx_mask_apply_workspace_size": (_sz, [_i64, _i64, _i32]),
    "onyx_mask_apply": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _sz, _vp]),
    "onyx_vocab_partial_workspace_size": (_sz, [_i64, _i64, _i32]),
    "onyx_vocab_partial_argmax": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _sz, _vp]),
    "onyx_combine_partials": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "onyx_masked_argmax_noalloc": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "onyx_masked_sample": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, ctypes.c_double, ctypes.c_double,
               ctypes.c_uint64, ctypes.c_uint64, _vp, _vp, _vp]),
    "onyx_dfa_state_masks": (
        _i32, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp]),
    "onyx_ipc_handle_bytes": (_sz, []),
    "onyx_exchange_buffer_bytes": (_sz, [_i32, _i64]),
    "onyx_ipc_alloc": (_i32, [_sz, ctypes.POINTER(_vp), _vp]),
    "onyx_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "onyx_ipc_close": (_i32, [_vp]),
    "onyx_ipc_free": (_i32, [_vp]),
    "onyx_vocab_exchange_argmax": (
        _i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _i32, _i32, ctypes.POINTER(_vp),
               _i64, _vp, _vp, _vp, _sz, _vp]),
}


class OnyxError(RuntimeError):
    """Base error of the onyx_b200 CUDA library boundary."""


class OnyxLibraryUnavailableError(OnyxError):
    """The compiled CUDA library is missing or cannot be loaded."""


class OnyxCallError(OnyxError):
    """A C-ABI call returned an error code."""

    def __init__(self, function: str, code: int, message: str) -> None:
        super().__init__(f"{function} failed: {message} (code {code})")
        self.function = function
        self.code = code


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and type the CUDA library; raise if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise OnyxLibraryUnavailableError(
                f"{target} is not built; run `python -c 'import __graft_entry__ as g; g.build()'`"
                " or `python onyx_b200/build_lib.py`"
            )
        try:
            lib = ctypes.CDLL(str(target))
        except OSError as exc:
            raise OnyxLibraryUnavailableError(f"cannot load {target}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.onyx_abi_version()
        if version != ABI_VERSION:
            raise OnyxLibraryUnavailableError(
                f"{target} has ABI version {version}; expected {ABI_VERSION}"
            )
        if path is None:
            _lib = lib
        return lib


def check(function: str, code: int) -> None:
    if code == OK:
        return
    lib = load()
    message = lib.onyx_error_string(code).decode()
    if code == ERR_CUDA:
        message += f"; cudaError {lib.onyx_last_cuda_error()}"
    raise OnyxCallError(function, code, message)


def set_option(option: int, value: int) -> None:
    """Set a process-wide library option (``OPTION_*``; diagnostic and test switches)."""
    check("onyx_set_option", load().onyx_set_option(int(option), int(value)))


def get_option(option: int) -> int:
    return int(load().onyx_get_option(int(option)))


class option_override:
    """Context manager: set library options for the duration of a block, then restore them.

    ``with option_override({OPTION_CLUSTER: 0}): ...``"""

    def __init__(self, values: dict[int, int]) -> None:
        self.values = dict(values)
        self.saved: dict[int, int] = {}

    def __enter__(self):
        for k, v in self.values.items():
            self.saved[k] = get_option(k)
            set_option(k, v)
        return self

    def __exit__(self, *exc):
        for k, v in self.saved.items():
            set_option(k, v)
