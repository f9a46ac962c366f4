"""Batched grammar-masked selection on B200: the torch-tensor face of the C ABI.

Every function here validates its tensors, picks the caller's current CUDA stream and
calls one entry point of ``libonyx_b200.so``; nothing is computed in Python or PyTorch and
nothing synchronises the device (results stay on the GPU). The per-row semantics are the
reference's single-row boundary applied to each row at once:

* masked row: valid values kept, -inf elsewhere
  (onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:145-186);
* greedy selection: lowest index of the maximum, NaN rejected
  (onyx_cuda/src/onyx_cuda/torch_backend.py:970-1007);
* speculative verify: accept while selection == draft, first mismatch -> replacement, full
  acceptance -> bonus selection of the final row
  (onyx_cuda/src/onyx_cuda/acceptance.py:96-132, grammar_acceptance.py:166-283,
  grammar_continuation.py:127-152).

Token masks are packed ``uint32`` words (``int32`` tensors are accepted as the same bits):
token ``t`` is valid iff bit ``t & 31`` of word ``t >> 5`` is set.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import _lib

__all__ = [
    "MaskedArgmaxResult",
    "SpecVerifyResult",
    "masked_argmax",
    "gather_masked_argmax",
    "spec_verify",
    "mask_apply",
    "vocab_partial_keys",
    "combine_partial_keys",
    "vocab_exchange_argmax",
    "mask_words",
    "dtype_code",
    "STATUS_EMPTY_MASK",
    "STATUS_ALL_NEG_INF",
    "STATUS_NAN_IN_SUPPORT",
    "STATUS_BAD_STATE",
    "STATUS_WAIT_TIMEOUT",
]

STATUS_EMPTY_MASK = _lib.STATUS_EMPTY_MASK
STATUS_ALL_NEG_INF = _lib.STATUS_ALL_NEG_INF
STATUS_NAN_IN_SUPPORT = _lib.STATUS_NAN_IN_SUPPORT
STATUS_BAD_STATE = _lib.STATUS_BAD_STATE
STATUS_WAIT_TIMEOUT = _lib.STATUS_WAIT_TIMEOUT

_DTYPE_CODES = {
    torch.float32: _lib.DTYPE_F32,
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float64: _lib.DTYPE_F64,
}
_MASK_DTYPES = (torch.int32, getattr(torch, "uint32", torch.int32))


def mask_words(vocab_size: int) -> int:
    """Number of uint32 words of one packed token mask row."""
    return (int(vocab_size) + 31) // 32


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported logits dtype {dtype}; expected float32/16, bfloat16, float64")


@dataclass(frozen=True)
class MaskedArgmaxResult:
    """Device tensors: ``token_ids`` int32[B] and ``status`` int32[B] (status bits)."""

    token_ids: torch.Tensor
    status: torch.Tensor


@dataclass(frozen=True)
class SpecVerifyResult:
    """Device tensors int32[B]: accepted draft count, correction token (-1: none), status."""

    accept_len: torch.Tensor
    correction: torch.Tensor
    status: torch.Tensor


# ---------------------------------------------------------------------------------------
# workspace: one zero-initialised buffer per (device, stream); kernels leave it zeroed
# ---------------------------------------------------------------------------------------
class _WorkspaceCache:
    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor | None:
        if nbytes == 0:
            return None
        key = (device.index, stream.cuda_stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 16)
                size = (size + 255) // 256 * 256
                with torch.cuda.stream(stream):
                    buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            return buf


_WORKSPACES = _WorkspaceCache()


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def _logits_2d(logits: torch.Tensor, name: str = "logits") -> torch.Tensor:
    _require_cuda(logits, name)
    dtype_code(logits.dtype)
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if logits.dim() != 2:
        raise ValueError(f"{name} must have shape [rows, vocab]; got {tuple(logits.shape)}")
    if logits.shape[1] <= 0:
        raise ValueError(f"{name} must have a non-empty vocabulary dimension")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    return logits


def _mask_2d(mask: torch.Tensor, rows: int, vocab: int, name: str = "bitmask") -> torch.Tensor:
    _require_cuda(mask, name)
    if mask.dtype not in _MASK_DTYPES:
        raise TypeError(f"{name} must be an int32/uint32 tensor of packed words; got {mask.dtype}")
    if mask.dim() == 1:
        mask = mask.unsqueeze(0)
    if mask.dim() != 2 or mask.shape[0] != rows or mask.shape[1] < mask_words(vocab):
        raise ValueError(
            f"{name} must have shape [{rows}, >={mask_words(vocab)}]; got {tuple(mask.shape)}"
        )
    if mask.stride(1) != 1:
        mask = mask.contiguous()
    return mask


def _same_device(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors[1:]:
        if t is not None and t.device != dev:
            raise ValueError(f"all tensors must be on {dev}; found {t.device}")
    return dev


def masked_argmax(logits: torch.Tensor, bitmask: torch.Tensor | None = None) -> MaskedArgmaxResult:
    """Masked greedy selection of every row of ``logits`` [B, V] (or one row [V]).

    ``bitmask`` [B, >=ceil(V/32)] packed words, or None to select over every column.
    """
    x = _logits_2d(logits)
    rows, vocab = x.shape
    m = _mask_2d(bitmask, rows, vocab) if bitmask is not None else None
    device = _same_device(x, *(t for t in (m,) if t is not None))
    idx = torch.empty(rows, dtype=torch.int32, device=device)
    status = torch.empty(rows, dtype=torch.int32, device=device)
    if rows == 0:
        return MaskedArgmaxResult(idx, status)
    lib = _lib.load()
    code = dtype_code(x.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = lib.onyx_masked_argmax_workspace_size(rows, vocab, code)
        ws = _WORKSPACES.get(device, stream, need)
        _lib.check(
            "onyx_masked_argmax",
            lib.onyx_masked_argmax(
                x.data_ptr(), code, rows, vocab, x.stride(0) if rows > 1 else vocab,
                _ptr(m), m.stride(0) if m is not None else 0,
                idx.data_ptr(), status.data_ptr(), _ptr(ws), 0 if ws is None else ws.numel(),
                stream.cuda_stream,
            ),
        )
    return MaskedArgmaxResult(idx, status)


def gather_masked_argmax(
    logits: torch.Tensor, table: torch.Tensor, state_ids: torch.Tensor
) -> MaskedArgmaxResult:
    """Row ``r`` is selected under mask row ``table[state_ids[r]]`` (per-DFA-state table)."""
    x = _logits_2d(logits)
    rows, vocab = x.shape
    _require_cuda(table, "table")
    if table.dtype not in _MASK_DTYPES or table.dim() != 2 or table.shape[1] < mask_words(vocab):
        raise ValueError(f"table must be int32/uint32 [states, >={mask_words(vocab)}]")
    if table.stride(1) != 1:
        table = table.contiguous()
    _require_cuda(state_ids, "state_ids")
    if state_ids.dtype != torch.int32 or state_ids.shape != (rows,):
        raise ValueError(f"state_ids must be int32 [{rows}]")
    state_ids = state_ids.contiguous()
    device = _same_device(x, table, state_ids)
    idx = torch.empty(rows, dtype=torch.int32, device=device)
    status = torch.empty(rows, dtype=torch.int32, device=device)
    if rows == 0:
        return MaskedArgmaxResult(idx, status)
    lib = _lib.load()
    code = dtype_code(x.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = lib.onyx_masked_argmax_workspace_size(rows, vocab, code)
        ws = _WORKSPACES.get(device, stream, need)
        _lib.check(
            "onyx_gather_masked_argmax",
            lib.onyx_gather_masked_argmax(
                x.data_ptr(), code, rows, vocab, x.stride(0) if rows > 1 else vocab,
                table.data_ptr(), table.shape[0], table.stride(0), state_ids.data_ptr(),
                idx.data_ptr(), status.data_ptr(), _ptr(ws), 0 if ws is None else ws.numel(),
                stream.cuda_stream,
            ),
        )
    return MaskedArgmaxResult(idx, status)


def spec_verify(
    logits: torch.Tensor, bitmasks: torch.Tensor, drafts: torch.Tensor, *, bonus: bool = True
) -> SpecVerifyResult:
    """Grammar-aware speculative verify.

    ``logits`` [B, G+1, V], ``bitmasks`` [B, G+1, >=ceil(V/32)], ``drafts`` int32 [B, G].
    Row ``i`` of entry ``b`` is judged under ``bitmasks[b, i]`` -- the grammar state reached
    by accepting drafts ``0..i-1``, which is the only state the reference ever inspects at
    position ``i`` (grammar_acceptance.py:196-259).
    """
    _require_cuda(logits, "logits")
    code = dtype_code(logits.dtype)
    if logits.dim() != 3:
        raise ValueError(f"logits must have shape [B, G+1, V]; got {tuple(logits.shape)}")
    batch, g1, vocab = logits.shape
    gamma = g1 - 1
    if gamma < 1:
        raise ValueError("speculative verify needs at least one draft token (G >= 1)")
    if logits.stride(2) != 1:
        logits = logits.contiguous()
    _require_cuda(bitmasks, "bitmasks")
    if (
        bitmasks.dtype not in _MASK_DTYPES
        or bitmasks.dim() != 3
        or bitmasks.shape[:2] != (batch, g1)
        or bitmasks.shape[2] < mask_words(vocab)
    ):
        raise ValueError(
            f"bitmasks must be int32/uint32 [{batch}, {g1}, >={mask_words(vocab)}]; "
            f"got {tuple(bitmasks.shape)}"
        )
    if bitmasks.stride(2) != 1:
        bitmasks = bitmasks.contiguous()
    _require_cuda(drafts, "drafts")
    if drafts.dtype != torch.int32 or drafts.shape != (batch, gamma):
        raise ValueError(f"drafts must be int32 [{batch}, {gamma}]")
    if drafts.stride(1) != 1:
        drafts = drafts.contiguous()
    device = _same_device(logits, bitmasks, drafts)
    accept = torch.empty(batch, dtype=torch.int32, device=device)
    corr = torch.empty(batch, dtype=torch.int32, device=device)
    status = torch.empty(batch, dtype=torch.int32, device=device)
    if batch == 0:
        return SpecVerifyResult(accept, corr, status)
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = lib.onyx_spec_verify_workspace_size(batch, gamma, vocab, code)
        ws = _WORKSPACES.get(device, stream, need)
        _lib.check(
            "onyx_spec_verify",
            lib.onyx_spec_verify(
                logits.data_ptr(), code, batch, gamma, vocab,
                logits.stride(0) if batch > 1 else g1 * logits.stride(1), logits.stride(1),
                bitmasks.data_ptr(),
                bitmasks.stride(0) if batch > 1 else g1 * bitmasks.stride(1),
                bitmasks.stride(1), drafts.data_ptr(), drafts.stride(0) if batch > 1 else gamma,
                1 if bonus else 0, accept.data_ptr(), corr.data_ptr(), status.data_ptr(),
                _ptr(ws), 0 if ws is None else ws.numel(), stream.cuda_stream,
            ),
        )
    return SpecVerifyResult(accept, corr, status)


def mask_apply(logits: torch.Tensor, bitmask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """New tensor with valid values bit-for-bit and -inf elsewhere, plus per-row status.

    The input is never modified and the result never aliases it
    (torch_grammar_mask.py:305-308).
    """
    squeeze = logits.dim() == 1 if isinstance(logits, torch.Tensor) else False
    x = _logits_2d(logits)
    rows, vocab = x.shape
    m = _mask_2d(bitmask, rows, vocab)
    device = _same_device(x, m)
    out = torch.empty((rows, vocab), dtype=x.dtype, device=device)
    status = torch.empty(rows, dtype=torch.int32, device=device)
    if rows:
        lib = _lib.load()
        code = dtype_code(x.dtype)
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device)
            need = lib.onyx_mask_apply_workspace_size(rows, vocab, code)
            ws = _WORKSPACES.get(device, stream, need)
            _lib.check(
                "onyx_mask_apply",
                lib.onyx_mask_apply(
                    x.data_ptr(), code, rows, vocab, x.stride(0) if rows > 1 else vocab,
                    m.data_ptr(), m.stride(0), out.data_ptr(), vocab, status.data_ptr(),
                    _ptr(ws), 0 if ws is None else ws.numel(), stream.cuda_stream,
                ),
            )
    if squeeze:
        return out.view(vocab), status
    return out, status


def vocab_partial_keys(
    logits_shard: torch.Tensor, mask_shard: torch.Tensor, col_offset: int
) -> torch.Tensor:
    """Packed (order, index) keys of this shard's columns, int64[B] (uint64 bit patterns).

    ``col_offset`` is the global id of the shard's first column (a multiple of 32); the
    mask words are the shard's own (``global_mask[:, col_offset//32 : ...]``).
    """
    x = _logits_2d(logits_shard, "logits_shard")
    rows, vocab = x.shape
    if x.dtype == torch.float64:
        raise TypeError("vocabulary-sharded selection supports float32/float16/bfloat16")
    if col_offset < 0 or col_offset % 32:
        raise ValueError("col_offset must be a non-negative multiple of 32")
    m = _mask_2d(mask_shard, rows, vocab, "mask_shard")
    device = _same_device(x, m)
    keys = torch.empty(rows, dtype=torch.int64, device=device)
    if rows == 0:
        return keys
    lib = _lib.load()
    code = dtype_code(x.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = lib.onyx_vocab_partial_workspace_size(rows, vocab, code)
        ws = _WORKSPACES.get(device, stream, need)
        _lib.check(
            "onyx_vocab_partial_argmax",
            lib.onyx_vocab_partial_argmax(
                x.data_ptr(), code, rows, vocab, x.stride(0) if rows > 1 else vocab,
                m.data_ptr(), m.stride(0), int(col_offset), keys.data_ptr(), _ptr(ws),
                0 if ws is None else ws.numel(), stream.cuda_stream,
            ),
        )
    return keys


def vocab_exchange_argmax(
    logits_shard: torch.Tensor, mask_shard: torch.Tensor, col_offset: int, *, world: int,
    rank: int, exchange_bases, rows_cap: int,
) -> MaskedArgmaxResult:
    """Full-vocabulary selections from this rank's shard, the keys exchanged through the
    ranks' NVLink-mapped exchange buffers (``exchange_bases``: a ctypes array of ``world``
    device pointers, this rank's own at ``rank``). Every rank makes the same calls in the
    same order. Use :class:`onyx_b200.vocab_parallel.PeerExchange` rather than calling
    this directly."""
    x = _logits_2d(logits_shard, "logits_shard")
    rows, vocab = x.shape
    if x.dtype == torch.float64:
        raise TypeError("vocabulary-sharded selection supports float32/float16/bfloat16")
    if col_offset < 0 or col_offset % 32:
        raise ValueError("col_offset must be a non-negative multiple of 32")
    if rows > rows_cap:
        raise ValueError(f"{rows} rows exceed the exchange buffers' capacity of {rows_cap}")
    m = _mask_2d(mask_shard, rows, vocab, "mask_shard")
    device = _same_device(x, m)
    idx = torch.empty(rows, dtype=torch.int32, device=device)
    status = torch.empty(rows, dtype=torch.int32, device=device)
    if rows == 0:
        return MaskedArgmaxResult(idx, status)
    lib = _lib.load()
    code = dtype_code(x.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        need = lib.onyx_vocab_partial_workspace_size(rows, vocab, code)
        ws = _WORKSPACES.get(device, stream, need)
        _lib.check(
            "onyx_vocab_exchange_argmax",
            lib.onyx_vocab_exchange_argmax(
                x.data_ptr(), code, rows, vocab, x.stride(0) if rows > 1 else vocab,
                m.data_ptr(), m.stride(0), int(col_offset), int(world), int(rank),
                exchange_bases, int(rows_cap), idx.data_ptr(), status.data_ptr(),
                _ptr(ws), 0 if ws is None else ws.numel(), stream.cuda_stream,
            ),
        )
    return MaskedArgmaxResult(idx, status)


def combine_partial_keys(keys: torch.Tensor) -> MaskedArgmaxResult:
    """Combine gathered shard keys ``[n_shards, B]`` into selections and status."""
    _require_cuda(keys, "keys")
    if keys.dtype != torch.int64 or keys.dim() != 2:
        raise ValueError("keys must be int64 [n_shards, rows]")
    keys = keys.contiguous()
    n, rows = keys.shape
    idx = torch.empty(rows, dtype=torch.int32, device=keys.device)
    status = torch.empty(rows, dtype=torch.int32, device=keys.device)
    if rows == 0:
        return MaskedArgmaxResult(idx, status)
    lib = _lib.load()
    with torch.cuda.device(keys.device):
        stream = torch.cuda.current_stream(keys.device)
        _lib.check(
            "onyx_combine_partials",
            lib.onyx_combine_partials(
                keys.data_ptr(), n, rows, idx.data_ptr(), status.data_ptr(), stream.cuda_stream
            ),
        )
    return MaskedArgmaxResult(idx, status)
