"""GPU mask producer: valid-token bitmasks of DFA states.

The reference rebuilds the valid-token set of the current grammar state on the CPU every
decoding step (``RegexConstraintCore::get_valid_token_ids``,
onyx_cuda/rust/src/regex_runtime.rs:129-145: every non-empty token whose byte walk through
the dense DFA from the state does not end dead). :class:`DfaMaskBuilder` does the same walk
on the GPU for any number of states in one launch (``onyx_dfa_state_masks``). The result is
either the mask row of one state, ready for :func:`onyx_b200.masked_argmax`, or the
per-state table that :func:`onyx_b200.gather_masked_argmax` reads by state id.

The transition table is the caller's: a dense ``[n_states, 256]`` next-state array with a
dead state, which is how regex-automata's dense DFA (the reference's regex engine) is laid
out.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from . import _lib

__all__ = ["pack_tokens", "dead_is_absorbing", "DfaMaskBuilder"]


def pack_tokens(tokens: Sequence[bytes]) -> tuple[np.ndarray, np.ndarray]:
    """CSR layout of a byte-string vocabulary: (bytes uint8[], offsets int64[V + 1])."""
    offsets = np.zeros(len(tokens) + 1, np.int64)
    offsets[1:] = np.cumsum([len(t) for t in tokens])
    data = np.frombuffer(b"".join(tokens), dtype=np.uint8).copy()
    return data, offsets


def dead_is_absorbing(trans: np.ndarray, dead: int) -> bool:
    """Whether every transition from ``dead`` returns to it (walks may then stop there)."""
    return bool(np.all(np.asarray(trans)[dead] == dead))


class DfaMaskBuilder:
    """A DFA and a vocabulary resident on one GPU; builds packed valid-token masks.

    ``trans``: int ``[n_states, 256]`` next-state ids; ``dead``: the dead state's id;
    ``tokens``: the vocabulary as byte strings (token id = position).
    """

    def __init__(self, trans, dead: int, tokens: Sequence[bytes],
                 device: torch.device | int | str | None = None) -> None:
        table = np.ascontiguousarray(np.asarray(trans), dtype=np.int32)
        if table.ndim != 2 or table.shape[1] != 256 or table.shape[0] < 1:
            raise ValueError("trans must be an int array of shape [n_states, 256]")
        if not 0 <= dead < table.shape[0]:
            raise ValueError(f"dead state {dead} outside [0, {table.shape[0]})")
        if len(tokens) < 1:
            raise ValueError("the vocabulary is empty")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device) if not isinstance(device, int) else torch.device(
            "cuda", device)
        if self.device.type != "cuda":
            raise ValueError("the mask producer runs on a CUDA device")
        data, offsets = pack_tokens(tokens)
        self.n_states = int(table.shape[0])
        self.dead = int(dead)
        self.absorbing = dead_is_absorbing(table, dead)
        self.vocab = len(tokens)
        self.words = (self.vocab + 31) // 32
        self._trans = torch.from_numpy(table).to(self.device)
        self._bytes = torch.from_numpy(data if data.size else np.zeros(1, np.uint8)).to(self.device)
        self._n_bytes = int(data.size)
        self._offsets = torch.from_numpy(offsets).to(self.device)

    def masks(self, states) -> torch.Tensor:
        """Packed masks of ``states`` (a sequence or int tensor of state ids): int32
        ``[len(states), ceil(V/32)]`` on the builder's device (uint32 bit patterns). A
        state id outside the table gives an all-zero row."""
        st = torch.as_tensor(states, dtype=torch.int32).reshape(-1).to(self.device)
        out = torch.empty((st.numel(), self.words), dtype=torch.int32, device=self.device)
        if st.numel() == 0:
            return out
        lib = _lib.load()
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            _lib.check(
                "onyx_dfa_state_masks",
                lib.onyx_dfa_state_masks(
                    self._trans.data_ptr(), self.n_states, self.dead, 1 if self.absorbing else 0,
                    st.data_ptr(), st.numel(), self._bytes.data_ptr(), self._n_bytes,
                    self._offsets.data_ptr(), self.vocab, out.data_ptr(), self.words,
                    stream.cuda_stream,
                ),
            )
        return out

    def table(self) -> torch.Tensor:
        """Masks of every state, row s = state s: the gather table."""
        return self.masks(torch.arange(self.n_states, dtype=torch.int32))
