"""The C-ABI library loads and exports every symbol its header declares (no GPU needed).

Only host-side functions are called here (ABI version, error strings, workspace sizing);
every compute entry point is exercised by the ``gpu`` tests.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from onyx_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "onyx_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(onyx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(cuda_lib):
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(raw, name), name


def test_abi_version_and_error_strings(cuda_lib):
    assert cuda_lib.onyx_abi_version() == _lib.ABI_VERSION
    for code in range(5):
        assert cuda_lib.onyx_error_string(code)
    assert b"unknown" in cuda_lib.onyx_error_string(99)


def test_workspace_sizes(cuda_lib):
    # a single segment needs no workspace
    assert cuda_lib.onyx_masked_argmax_workspace_size(4, 1000, _lib.DTYPE_BF16) == 0
    # 64 rows of 128,256 bf16 split into segments: partials + counters, 256-aligned
    n = cuda_lib.onyx_masked_argmax_workspace_size(64, 128256, _lib.DTYPE_BF16)
    assert n > 0 and n % 256 == 0
    assert cuda_lib.onyx_spec_verify_workspace_size(32, 4, 151936, _lib.DTYPE_BF16) > 0
    assert cuda_lib.onyx_spec_verify_workspace_size(32, 0, 151936, _lib.DTYPE_BF16) == 0
    assert cuda_lib.onyx_vocab_partial_workspace_size(8, 1000, _lib.DTYPE_F64) == 0
    assert cuda_lib.onyx_masked_argmax_workspace_size(4, 1000, 17) == 0


def test_argument_errors_are_reported_before_any_launch(cuda_lib):
    # every call below is rejected on the host, so no CUDA call is made
    assert cuda_lib.onyx_masked_argmax(None, 9, 1, 10, 10, None, 0, None, None, None, 0, None) == \
        _lib.ERR_UNSUPPORTED_DTYPE
    assert cuda_lib.onyx_masked_argmax(None, 0, 1, 0, 0, None, 0, None, None, None, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert cuda_lib.onyx_masked_argmax(None, 0, 0, 10, 10, None, 0, None, None, None, 0, None) == \
        _lib.OK  # zero rows: nothing to do
    assert cuda_lib.onyx_spec_verify(
        None, 2, 1, 0, 10, 0, 10, None, 0, 1, None, 0, 1, None, None, None, None, 0, None
    ) == _lib.ERR_INVALID_ARGUMENT  # gamma 0: the reference rejects an empty proposal
    assert cuda_lib.onyx_vocab_partial_argmax(
        None, 3, 1, 10, 10, None, 1, 0, None, None, 0, None
    ) == _lib.ERR_UNSUPPORTED_DTYPE
    assert cuda_lib.onyx_combine_partials(None, 0, 1, None, None, None) == \
        _lib.ERR_INVALID_ARGUMENT


def test_options_round_trip_and_reject_bad_values(cuda_lib):
    saved = {k: _lib.get_option(k) for k in range(4)}
    try:
        assert saved[_lib.OPTION_CLUSTER] in (0, 1) and saved[_lib.OPTION_PDL] in (0, 1)
        for k, v in ((_lib.OPTION_CLUSTER, 0), (_lib.OPTION_PDL, 0), (_lib.OPTION_SAMPLE_FORM, -1),
                     (_lib.OPTION_TEST_WITHHELD_KEY_BYTES, 8)):
            _lib.set_option(k, v)
            assert _lib.get_option(k) == v
        for k, v in ((_lib.OPTION_CLUSTER, 2), (_lib.OPTION_PDL, -1), (_lib.OPTION_SAMPLE_FORM, 17),
                     (_lib.OPTION_TEST_WITHHELD_KEY_BYTES, -1), (4, 0), (-1, 0)):
            assert cuda_lib.onyx_set_option(k, v) == _lib.ERR_INVALID_ARGUMENT
        assert cuda_lib.onyx_get_option(4) == -1
        with _lib.option_override({_lib.OPTION_CLUSTER: 1}):
            assert _lib.get_option(_lib.OPTION_CLUSTER) == 1
        assert _lib.get_option(_lib.OPTION_CLUSTER) == 0
    finally:
        for k, v in saved.items():
            _lib.set_option(k, v)


def test_missing_library_fails_loudly(tmp_path):
    import pytest

    with pytest.raises(_lib.OnyxLibraryUnavailableError):
        _lib.load(tmp_path / "libonyx_b200.so")
