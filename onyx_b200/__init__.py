"""onyx_b200: B200-native (sm_100a) grammar-constrained selection for Onyx.

The hot path of bayareahomelander/Onyx's constrained decoding -- grammar-masked greedy
selection, grammar-aware speculative verify, and DFA-state mask gather -- as hand-written
CUDA behind a C ABI (``include/onyx_b200.h``, ``libonyx_b200.so``), with the reference's
Python boundary kept as a drop-in:

* :mod:`onyx_b200.torch_grammar_mask` -- ``create_cuda_grammar_logit_mask`` /
  ``TorchCUDAGrammarLogitMask`` (``apply``, ``apply_with_timing``);
* :mod:`onyx_b200.torch_backend` -- ``select_cuda_argmax``;
* :mod:`onyx_b200.masked_selection` -- batched ``masked_argmax``, ``spec_verify``,
  ``gather_masked_argmax``, ``mask_apply`` on torch tensors;
* :mod:`onyx_b200.vocab_parallel` -- batch- and vocabulary-sharded multi-GPU selection.
"""

from . import bitmask
from .dfa_masks import DfaMaskBuilder
from .sampling import TemperatureTopPSelection, create_cuda_sampler, masked_sample
from ._lib import OnyxCallError, OnyxError, OnyxLibraryUnavailableError
from .masked_selection import (
    STATUS_ALL_NEG_INF,
    STATUS_BAD_STATE,
    STATUS_EMPTY_MASK,
    STATUS_NAN_IN_SUPPORT,
    STATUS_WAIT_TIMEOUT,
    MaskedArgmaxResult,
    SpecVerifyResult,
    combine_partial_keys,
    gather_masked_argmax,
    mask_apply,
    masked_argmax,
    spec_verify,
    vocab_partial_keys,
)
from .torch_backend import select_cuda_argmax, select_masked_cuda_argmax
from .torch_grammar_mask import TorchCUDAGrammarLogitMask, create_cuda_grammar_logit_mask

__all__ = [
    "bitmask",
    "OnyxError",
    "OnyxCallError",
    "OnyxLibraryUnavailableError",
    "MaskedArgmaxResult",
    "SpecVerifyResult",
    "masked_argmax",
    "gather_masked_argmax",
    "spec_verify",
    "mask_apply",
    "vocab_partial_keys",
    "combine_partial_keys",
    "select_cuda_argmax",
    "select_masked_cuda_argmax",
    "create_cuda_grammar_logit_mask",
    "TorchCUDAGrammarLogitMask",
    "STATUS_EMPTY_MASK",
    "STATUS_ALL_NEG_INF",
    "STATUS_NAN_IN_SUPPORT",
    "STATUS_BAD_STATE",
    "STATUS_WAIT_TIMEOUT",
    "DfaMaskBuilder",
    "TemperatureTopPSelection",
    "create_cuda_sampler",
    "masked_sample",
]
