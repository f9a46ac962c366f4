/*
 * onyx_b200 -- C ABI of the B200 (sm_100a) grammar-masked selection library.
 *
 * Plain pointers and sizes only: every buffer is caller-owned device memory, `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream), and no call allocates,
 * synchronises or retains a pointer. Launches are asynchronous; per-row data errors are
 * reported through the status outputs, launch/argument errors through the return code.
 *
 * Token-mask layout (the bitmask convention of this library): token id t of a row is valid
 * iff bit (t & 31) of word (t >> 5) is set, words little-endian uint32, W = ceil(V/32)
 * words per row, bits at ids >= V ignored. The reference passes the same set as a sorted
 * tuple of ids (onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:69-86, :399-422).
 *
 * Selection semantics (shared by every entry point): the masked row keeps valid values and
 * is -inf elsewhere (torch_grammar_mask.py:145-186); the selected id is the lowest index
 * holding the maximum under float comparison (-0.0 == +0.0, +inf ties resolve low;
 * onyx_cuda/src/onyx_cuda/torch_backend.py:970-1007, generation.py:212-224).
 *
 * Workspace: entry points that split one row over several CTAs need a caller-owned device
 * workspace of the size returned by the matching *_workspace_size function (0 means none
 * is needed and NULL may be passed). It must be 256-byte aligned and zero-filled before its
 * first use; every call leaves it zero-filled again. Calls that may run concurrently (other
 * streams) need separate workspaces.
 */
#ifndef ONYX_B200_H_
#define ONYX_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ONYX_ABI_VERSION 1

#if defined(__GNUC__)
#define ONYX_API __attribute__((visibility("default")))
#else
#define ONYX_API
#endif

/* dtype codes */
#define ONYX_DTYPE_F32 0
#define ONYX_DTYPE_F16 1
#define ONYX_DTYPE_BF16 2
#define ONYX_DTYPE_F64 3

/* return codes */
#define ONYX_OK 0
#define ONYX_ERR_INVALID_ARGUMENT 1
#define ONYX_ERR_UNSUPPORTED_DTYPE 2
#define ONYX_ERR_WORKSPACE 3
#define ONYX_ERR_CUDA 4
#define ONYX_ERR_SCRATCH_LIMIT 5 /* onyx_masked_argmax_noalloc: beyond its fixed scratch */

/* size of the per-device scratch array of onyx_masked_argmax_noalloc */
#define ONYX_NOALLOC_SCRATCH_BYTES (1u << 20)

/* per-row status bits */
#define ONYX_STATUS_EMPTY_MASK 1u     /* no valid token: grammar no-decision
                                         (grammar_selection.py:122-127) */
#define ONYX_STATUS_ALL_NEG_INF 2u    /* valid tokens exist but every value is -inf:
                                         rejected by torch_grammar_mask.py:182-185 */
#define ONYX_STATUS_NAN_IN_SUPPORT 4u /* a valid value is NaN: rejected by
                                         torch_backend.py:991-996 */
#define ONYX_STATUS_BAD_STATE 8u      /* gather: DFA state id outside the table */
#define ONYX_STATUS_WAIT_TIMEOUT 16u  /* a bounded wait inside the kernel for the row's
                                         partial results gave up (a hardware fault): the
                                         row's output is not valid */

ONYX_API int onyx_abi_version(void);
ONYX_API const char* onyx_error_string(int code);
/* cudaError_t of the last failed launch on this host thread */
ONYX_API int onyx_last_cuda_error(void);

/*
 * Process-wide diagnostic and test options. None is needed in normal use; each starts from
 * an environment variable read once, at the first call that uses any option, and changes
 * only through onyx_set_option (which returns ONYX_ERR_INVALID_ARGUMENT for an unknown id
 * or value). Options apply to launches made after the change. No counterpart in the
 * reference (its selection is plain PyTorch).
 *   CLUSTER      1: rows that fit one thread-block cluster use the cluster kernel;
 *                0: the global-ticket merge instead (ONYX_B200_CLUSTER, default 1).
 *   PDL          1: launches allow programmatic dependent launch (ONYX_B200_PDL, default 1).
 *   SAMPLE_FORM  masked sampling: 0 the cluster form with the cluster size chosen from the
 *                batch, -1 the one-CTA form, k in [1, 16] clusters of k CTAs
 *                (ONYX_B200_SAMPLE_FORM: "single" or "cluster:<k>", default 0).
 *   TEST_WITHHELD_KEY_BYTES  test hook, 0 in normal use: rank 0 of a cluster expects this
 *                many key bytes beyond those its CTAs send, so its bounded wait runs out
 *                and the rows report ONYX_STATUS_WAIT_TIMEOUT. Set only by tests.
 */
#define ONYX_OPTION_CLUSTER 0
#define ONYX_OPTION_PDL 1
#define ONYX_OPTION_SAMPLE_FORM 2
#define ONYX_OPTION_TEST_WITHHELD_KEY_BYTES 3
#define ONYX_OPTION_COUNT 4
ONYX_API int onyx_set_option(int option, int64_t value);
ONYX_API int64_t onyx_get_option(int option);

/*
 * Masked greedy selection over `rows` rows of `vocab` logits.
 * Replaces TorchCUDAGrammarLogitMask.apply + select_cuda_argmax for a whole batch
 * (onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:69-86 and torch_backend.py:970-1007).
 * logits: rows x vocab, row r at logits + r*row_stride elements (dtype code).
 * mask:   rows x mask_stride words, or NULL to select over every column (the plain
 *         select_cuda_argmax contract: NaN rejected, first maximum).
 * out_idx[r]: selected id (int32), -1 on EMPTY_MASK / NAN_IN_SUPPORT; on ALL_NEG_INF the
 *             lowest valid id. out_status[r]: status bits.
 */
ONYX_API size_t onyx_masked_argmax_workspace_size(int64_t rows, int64_t vocab, int dtype);
ONYX_API int onyx_masked_argmax(const void* logits, int dtype, int64_t rows, int64_t vocab,
                       int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                       int32_t* out_idx, uint32_t* out_status, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Fused per-DFA-state mask-table gather + masked greedy selection: row r uses mask row
 * table[state_ids[r]] (n_states rows of table_stride words). The table is the reference's
 * valid-id scan (onyx_cuda/rust/src/regex_runtime.rs:129-145) precomputed per state, so this
 * replaces get_valid_token_ids + apply + select for a batch. Ids outside [0, n_states)
 * give BAD_STATE. Uses the masked-argmax workspace size.
 */
ONYX_API int onyx_gather_masked_argmax(const void* logits, int dtype, int64_t rows, int64_t vocab,
                              int64_t row_stride, const uint32_t* table, int64_t n_states,
                              int64_t table_stride, const int32_t* state_ids, int32_t* out_idx,
                              uint32_t* out_status, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * Grammar-aware speculative verify of `batch` entries with `gamma` draft tokens each.
 * Row (b,i), i in [0,gamma], is logits + b*batch_stride + i*row_stride with mask
 * masks + b*mask_batch_stride + i*mask_row_stride; drafts[b*draft_stride + i], i < gamma.
 * accept_len[b] = first i < gamma whose masked selection differs from the draft (else
 * gamma); correction[b] = that selection, or on full acceptance the selection of row gamma
 * when bonus != 0 (onyx_cuda grammar_continuation.py:127-152), else -1 (macOS loop without
 * bonus, onyx/speculative.py:545-608). A row with a status bit ends the decision at that
 * row: accept_len = i, correction = -1, out_status[b] = the row's bits
 * (grammar_acceptance.py:196-283). Replaces decide_match_replace_acceptance /
 * decide_grammar_masked_target_acceptance (acceptance.py:96-132, grammar_acceptance.py:166).
 * gamma in [1, 255].
 */
ONYX_API size_t onyx_spec_verify_workspace_size(int64_t batch, int64_t gamma, int64_t vocab, int dtype);
ONYX_API int onyx_spec_verify(const void* logits, int dtype, int64_t batch, int64_t gamma, int64_t vocab,
                     int64_t batch_stride, int64_t row_stride, const uint32_t* masks,
                     int64_t mask_batch_stride, int64_t mask_row_stride, const int32_t* drafts,
                     int64_t draft_stride, int bonus, int32_t* accept_len, int32_t* correction,
                     uint32_t* out_status, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * Materialise masked rows: out = valid values bit-for-bit, -inf elsewhere; out_status gets
 * EMPTY_MASK / ALL_NEG_INF (TorchCUDAGrammarLogitMask._apply_device_indices,
 * torch_grammar_mask.py:145-186). `out` must not alias `logits`.
 */
ONYX_API size_t onyx_mask_apply_workspace_size(int64_t rows, int64_t vocab, int dtype);
ONYX_API int onyx_mask_apply(const void* logits, int dtype, int64_t rows, int64_t vocab,
                    int64_t row_stride, const uint32_t* mask, int64_t mask_stride, void* out,
                    int64_t out_stride, uint32_t* out_status, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Vocabulary-parallel selection, step 1: this rank's column shard [col_offset,
 * col_offset + shard_vocab) of every row (col_offset a multiple of 32; the mask words are
 * the shard's own). out_keys[r] packs (order code of the maximum << 32) | (0xFFFFFFFF -
 * global id); 0 means no valid token in the shard. Gather the keys of all shards (e.g.
 * NCCL all-gather) and combine with onyx_combine_partials. Not for f64.
 * No counterpart in the reference (single device only); it splits select_cuda_argmax's
 * reduction over GPUs with identical results.
 */
ONYX_API size_t onyx_vocab_partial_workspace_size(int64_t rows, int64_t shard_vocab, int dtype);
ONYX_API int onyx_vocab_partial_argmax(const void* logits, int dtype, int64_t rows, int64_t shard_vocab,
                              int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                              int64_t col_offset, uint64_t* out_keys, void* workspace,
                              size_t workspace_bytes, void* stream);
/* step 2: keys[part*rows + r] for n_parts shards -> out_idx / out_status as masked argmax */
ONYX_API int onyx_combine_partials(const uint64_t* keys, int64_t n_parts, int64_t rows, int32_t* out_idx,
                          uint32_t* out_status, void* stream);

/*
 * Masked temperature / top-p sampling, one draw per row. The distribution and the kept
 * (top-p) set are the reference's (onyx_cuda/src/onyx_cuda/selection.py,
 * _filtered_reference_weights, float64): over the valid ids, any +inf shares the mass
 * equally among the +inf ids, else weights exp((v - max) / temperature); ranked by
 * (-probability, id), the shortest prefix reaching top_p is kept. The draw of row r is
 * Philox4x32-10 with key `seed` and counter (call, r), as a 53-bit double u; the sampled id
 * is the first kept id in id order whose cumulative kept probability exceeds u times the
 * kept total. Same arguments, same outputs. Status bits as for onyx_masked_argmax
 * (EMPTY_MASK, ALL_NEG_INF, NAN_IN_SUPPORT; the id is -1 with any of them).
 * temperature finite and > 0, 0 < top_p <= 1; bf16 / f16 / f32.
 */
ONYX_API int onyx_masked_sample(const void* logits, int dtype, int64_t rows, int64_t vocab,
                                int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                                double temperature, double top_p, uint64_t seed, uint64_t call,
                                int32_t* out_idx, uint32_t* out_status, void* stream);

/*
 * Valid-token bitmasks of DFA states (the mask producer): row r of `out` (out_stride >=
 * ceil(vocab/32) words) is the packed mask of states[r] -- bit t set iff token t is
 * non-empty and walking its bytes through `trans` ([n_states][256] next-state ids) from
 * states[r] does not end in `dead`. Restates get_valid_token_ids,
 * onyx_cuda/rust/src/regex_runtime.rs:129-145 (transition fold :197-201), for every row in
 * one launch; building it for every reachable state gives the table that
 * onyx_gather_masked_argmax reads. Tokens are CSR: tok_bytes[n_bytes], tok_offsets[vocab+1].
 * `dead_absorbing` nonzero promises every transition from `dead` returns to it (true of
 * regex-automata's dense DFAs) and lets walks stop there. Out-of-range transitions count as
 * dead, out-of-range state ids give empty rows, and offsets outside the byte array give empty
 * tokens, so malformed input is never read out of bounds. n_states is at most 2^23 (8 GB
 * of table); beyond it the call returns ONYX_ERR_INVALID_ARGUMENT.
 */
ONYX_API int onyx_dfa_state_masks(const int32_t* trans, int32_t n_states, int32_t dead,
                                  int dead_absorbing, const int32_t* states, int64_t rows,
                                  const uint8_t* tok_bytes, int64_t n_bytes,
                                  const int64_t* tok_offsets, int64_t vocab, uint32_t* out,
                                  int64_t out_stride, void* stream);

/*
 * Vocabulary-parallel selection with the key exchange over NVLink peer memory instead of a
 * collective library call: the shard-key kernel writes each row's key straight into every
 * rank's exchange buffer, and one small kernel raises this rank's flag in every buffer
 * (system-scope release), waits until every rank's flag in its own buffer reaches this
 * call's number (bounded: rows get ONYX_STATUS_WAIT_TIMEOUT if it gives up) and combines.
 * Replaces the all-gather + onyx_combine_partials pair above with identical results. No
 * counterpart in the reference (single device only; torch_backend.py:970-1007 is the
 * selection it distributes).
 *
 * Exchange buffers: every rank allocates onyx_exchange_buffer_bytes(world, rows_cap) with
 * onyx_ipc_alloc, shares the onyx_ipc_handle_bytes()-byte handle with the other ranks (any
 * host channel), and opens theirs with onyx_ipc_open. `exchange_bases[i]` is rank i's
 * buffer as mapped in this process (its own at [rank]). Every rank makes the same calls in
 * the same order; each rank's buffer counts its finished calls on the device, so the calls
 * may be captured in a CUDA graph and replayed. world <= 8.
 */
ONYX_API size_t onyx_ipc_handle_bytes(void);
ONYX_API size_t onyx_exchange_buffer_bytes(int world, int64_t rows_cap);
ONYX_API int onyx_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out);
ONYX_API int onyx_ipc_open(const void* handle, void** dev_ptr);
ONYX_API int onyx_ipc_close(void* dev_ptr);
ONYX_API int onyx_ipc_free(void* dev_ptr);
ONYX_API int onyx_vocab_exchange_argmax(const void* logits, int dtype, int64_t rows,
                                        int64_t shard_vocab, int64_t row_stride,
                                        const uint32_t* mask, int64_t mask_stride,
                                        int64_t col_offset, int world, int rank,
                                        void* const* exchange_bases, int64_t rows_cap,
                                        int32_t* out_idx, uint32_t* out_status,
                                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Allocation-free masked greedy selection. No counterpart in the reference: it is the
 * onyx_masked_argmax contract for callers that cannot allocate device memory when they
 * call -- a serving process whose GPU memory is reserved up front by its own pool, a
 * foreign-language binding that only receives pointers to buffers allocated elsewhere, or
 * code where an allocation would synchronise or fail -- and so cannot pass a workspace.
 * The caller passes only inputs and outputs (same meaning as onyx_masked_argmax).
 *
 * Rows that fit one thread-block cluster (up to 8 x 16 warp segments: 262,144 columns of a
 * 16-byte aligned 16-bit row, 131,072 of f32, 131,072 of an unaligned row) combine inside
 * the cluster and use no scratch, unless ONYX_OPTION_CLUSTER is off. Longer rows, and f64
 * rows, keep their partials and tickets in a fixed scratch array compiled into the
 * library: ONYX_NOALLOC_SCRATCH_BYTES (1 MiB) held on every GPU that loads the library
 * until the process exits. Such a request needs 4 bytes per row (rounded up to 256) plus
 * 16 bytes per row per CTA; a CTA covers 16,384 columns of a 16-byte aligned 16-bit row,
 * 8,192 columns of an aligned f32 row, and 8,192 columns otherwise (unaligned rows, f64).
 * A request needing more returns ONYX_ERR_SCRATCH_LIMIT without launching anything. The
 * call allocates nothing: the first call that needs the scratch in a CUDA context looks up
 * its address (cudaGetSymbolAddress) and keeps it for that context, so make that first call
 * (for the primary context, the first on each device) before any stream capture; every
 * call that uses the scratch clears its tickets with cudaMemsetAsync on `stream`. All calls
 * in a context share the one array, so calls that can overlap on the GPU (other streams or
 * host threads) race and must be serialised by the caller.
 */
ONYX_API int onyx_masked_argmax_noalloc(const void* logits, int dtype, int64_t rows,
                                        int64_t vocab, int64_t row_stride, const uint32_t* mask,
                                        int64_t mask_stride, int32_t* out_idx,
                                        uint32_t* out_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ONYX_B200_H_ */
