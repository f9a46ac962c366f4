/*
 * CPU oracle for the grammar-masked selection path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, the smoke entry
 * point and the CPU-baseline leg of bench.py load it. The CUDA library in
 * onyx_b200/ never links or calls it.
 *
 * It restates, as plain scalar C, the semantics of the reference
 * (bayareahomelander/Onyx, onyx_cuda package):
 *
 *   mask      onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:145-186
 *             allowed logits are kept bit-for-bit, everything else becomes
 *             -inf; a support that is entirely -inf is rejected (:182-185).
 *   select    onyx_cuda/src/onyx_cuda/generation.py:212-224 (CPU) and
 *             onyx_cuda/src/onyx_cuda/torch_backend.py:970-1007 (CUDA):
 *             first (lowest-index) maximum, NaN anywhere in the masked row
 *             rejected. Floats compare as floats, so -0.0 == +0.0 and equal
 *             maxima resolve to the lowest index.
 *   verify    onyx_cuda/src/onyx_cuda/acceptance.py:115-132 and
 *             grammar_acceptance.py:196-283: accept while select(row_i) equals
 *             draft_i; the first mismatch yields the replacement; an empty
 *             support at position i is a no-decision at i.
 *   bonus     onyx_cuda/src/onyx_cuda/grammar_continuation.py:127-152: on full
 *             acceptance the correction is the masked selection of the final
 *             row (macOS loop onyx/speculative.py:545-608 has no bonus).
 *
 * The bitmask convention (token id -> word id>>5, bit id&31, LSB first) is the
 * one the CUDA library uses; the reference passes sorted sparse ids, and
 * packing those ids into this layout is exactly the set membership test of
 * the reference's list masks (tests/test_grammar_selection.py:791-798).
 *
 * The oracle deliberately walks every row element by element with an explicit
 * "found / best / best index" state (the shape of select_highest_logit),
 * rather than the packed-key reduction the GPU kernels use, so that the two are
 * independent formulations of the same contract.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* dtype codes shared with the CUDA library's C-ABI */
enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2, OR_F64 = 3 };

/* per-row status bits shared with the CUDA library's C-ABI */
enum {
    OR_EMPTY_MASK = 1u,     /* no valid token: grammar no-decision */
    OR_ALL_NEG_INF = 2u,    /* support exists but every value is -inf */
    OR_NAN_IN_SUPPORT = 4u, /* selector rejects NaN */
    OR_BAD_STATE = 8u       /* DFA state id outside the table */
};

static double load_as_double(const void* base, int dtype, int64_t i) {
    switch (dtype) {
    case OR_F32: return (double)((const float*)base)[i];
    case OR_F64: return ((const double*)base)[i];
    case OR_BF16: {
        uint32_t u = (uint32_t)((const uint16_t*)base)[i] << 16;
        float f;
        memcpy(&f, &u, 4);
        return (double)f;
    }
    case OR_F16: {
        _Float16 h;
        memcpy(&h, (const uint16_t*)base + i, 2);
        return (double)h;
    }
    }
    return NAN;
}

static int64_t elem_size(int dtype) {
    switch (dtype) {
    case OR_F32: return 4;
    case OR_F64: return 8;
    default: return 2;
    }
}

static inline int mask_bit(const uint32_t* mask_row, int64_t i) {
    return (int)((mask_row[i >> 5] >> (i & 31)) & 1u);
}

/* One row: select_highest_logit over the masked row, with the mask checks. */
static void select_row(const void* row, int dtype, int64_t V, const uint32_t* mask_row,
                       int32_t* out_idx, uint32_t* out_status) {
    int found = 0, saw_nan = 0;
    double best = 0.0;
    int64_t best_i = -1;
    for (int64_t i = 0; i < V; ++i) {
        if (mask_row && !mask_bit(mask_row, i)) continue;
        double v = load_as_double(row, dtype, i);
        if (isnan(v)) {
            saw_nan = 1;
            continue;
        }
        if (!found || v > best) {
            best = v;
            best_i = i;
            found = 1;
        }
    }
    if (!found && !saw_nan) {
        *out_idx = -1;
        *out_status = OR_EMPTY_MASK;
    } else if (saw_nan) {
        *out_idx = -1;
        *out_status = OR_NAN_IN_SUPPORT;
    } else {
        *out_idx = (int32_t)best_i;
        *out_status = (best == -INFINITY) ? OR_ALL_NEG_INF : 0u;
    }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

/* masked argmax over B rows; mask may be NULL (plain first-max argmax) */
int oracle_masked_argmax(const void* logits, int dtype, int64_t B, int64_t V, int64_t row_stride,
                         const uint32_t* mask, int64_t mask_stride, int32_t* out_idx,
                         uint32_t* out_status, int nthreads) {
    if (B < 0 || V <= 0) return 1;
    set_threads(nthreads);
    const char* base = (const char*)logits;
    int64_t es = elem_size(dtype);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t r = 0; r < B; ++r) {
        select_row(base + r * row_stride * es, dtype, V, mask ? mask + r * mask_stride : NULL,
                   &out_idx[r], &out_status[r]);
    }
    return 0;
}

/* gather mask rows from a per-DFA-state table by state id, then masked argmax */
int oracle_gather_masked_argmax(const void* logits, int dtype, int64_t B, int64_t V,
                                int64_t row_stride, const uint32_t* table, int64_t n_states,
                                int64_t table_stride, const int32_t* state_ids, int32_t* out_idx,
                                uint32_t* out_status, int nthreads) {
    if (B < 0 || V <= 0) return 1;
    set_threads(nthreads);
    const char* base = (const char*)logits;
    int64_t es = elem_size(dtype);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t r = 0; r < B; ++r) {
        int32_t s = state_ids[r];
        if (s < 0 || (int64_t)s >= n_states) {
            out_idx[r] = -1;
            out_status[r] = OR_BAD_STATE;
            continue;
        }
        select_row(base + r * row_stride * es, dtype, V, table + (int64_t)s * table_stride,
                   &out_idx[r], &out_status[r]);
    }
    return 0;
}

/*
 * Grammar-aware speculative verify over B batch rows of G+1 target rows.
 * Row (b,i) lives at logits + b*batch_stride + i*row_stride (elements) and its
 * mask at masks + b*mask_batch_stride + i*mask_row_stride (words).
 * Outputs: accept_len[b] in [0,G]; correction[b] = replacement (mismatch),
 * bonus (full acceptance and bonus != 0) or -1; status[b] = status bits of
 * the row that ended the decision (0 when it decided normally).
 * Also writes the per-row selections into row_idx/row_status when non-NULL.
 */
int oracle_spec_verify(const void* logits, int dtype, int64_t B, int64_t G, int64_t V,
                       int64_t batch_stride, int64_t row_stride, const uint32_t* masks,
                       int64_t mask_batch_stride, int64_t mask_row_stride, const int32_t* drafts,
                       int64_t draft_stride, int bonus, int32_t* accept_len, int32_t* correction,
                       uint32_t* status, int nthreads) {
    if (B < 0 || G < 0 || V <= 0) return 1;
    set_threads(nthreads);
    const char* base = (const char*)logits;
    int64_t es = elem_size(dtype);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b) {
        int32_t acc = (int32_t)G, corr = -1;
        uint32_t st = 0;
        int decided = 0;
        for (int64_t i = 0; i < G && !decided; ++i) {
            int32_t sel;
            uint32_t rs;
            select_row(base + (b * batch_stride + i * row_stride) * es, dtype, V,
                       masks + b * mask_batch_stride + i * mask_row_stride, &sel, &rs);
            if (rs & (OR_EMPTY_MASK | OR_NAN_IN_SUPPORT | OR_ALL_NEG_INF)) {
                acc = (int32_t)i;
                corr = -1;
                st = rs;
                decided = 1;
            } else if (sel != drafts[b * draft_stride + i]) {
                acc = (int32_t)i;
                corr = sel;
                decided = 1;
            }
        }
        if (!decided && bonus) {
            int32_t sel;
            uint32_t rs;
            select_row(base + (b * batch_stride + G * row_stride) * es, dtype, V,
                       masks + b * mask_batch_stride + G * mask_row_stride, &sel, &rs);
            if (rs & (OR_EMPTY_MASK | OR_NAN_IN_SUPPORT | OR_ALL_NEG_INF)) {
                corr = -1;
                st = rs;
            } else {
                corr = sel;
            }
        }
        accept_len[b] = acc;
        correction[b] = corr;
        status[b] = st;
    }
    return 0;
}

/*
 * Materialise the masked rows: out[r,i] = in[r,i] (bit-for-bit) if bit set,
 * else -inf. status[r] gets OR_EMPTY_MASK / OR_ALL_NEG_INF as the reference's
 * apply() would reject (torch_grammar_mask.py:182-185, :405-406).
 */
int oracle_mask_apply(const void* logits, int dtype, int64_t B, int64_t V, int64_t row_stride,
                      const uint32_t* mask, int64_t mask_stride, void* out, int64_t out_stride,
                      uint32_t* out_status) {
    int64_t es = elem_size(dtype);
    for (int64_t r = 0; r < B; ++r) {
        const char* src = (const char*)logits + r * row_stride * es;
        char* dst = (char*)out + r * out_stride * es;
        const uint32_t* m = mask + r * mask_stride;
        int any = 0, all_ninf = 1;
        for (int64_t i = 0; i < V; ++i) {
            if (mask_bit(m, i)) {
                memcpy(dst + i * es, src + i * es, (size_t)es);
                any = 1;
                double v = load_as_double(src, dtype, i);
                if (!(v == -INFINITY)) all_ninf = 0;
            } else {
                switch (dtype) {
                case OR_F32: { float x = -INFINITY; memcpy(dst + i * es, &x, 4); break; }
                case OR_F64: { double x = -INFINITY; memcpy(dst + i * es, &x, 8); break; }
                case OR_BF16: { uint16_t x = 0xFF80u; memcpy(dst + i * es, &x, 2); break; }
                case OR_F16: { uint16_t x = 0xFC00u; memcpy(dst + i * es, &x, 2); break; }
                }
            }
        }
        out_status[r] = !any ? OR_EMPTY_MASK : (all_ninf ? OR_ALL_NEG_INF : 0u);
    }
    return 0;
}

/*
 * Vocabulary-parallel form: each shard holds columns [col_offset, col_offset+Vs)
 * of every row (mask words for the same columns, col_offset a multiple of 32).
 * The shard result is (found, nan, best value, best global index); combining
 * shards in increasing col_offset order with "strictly greater wins" gives the
 * same answer as the unsharded select.
 */
typedef struct {
    int32_t found, nan;
    double best;
    int64_t idx;
} oracle_partial;

int oracle_vocab_shard_select(const void* logits, int dtype, int64_t B, int64_t Vs,
                              int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                              int64_t col_offset, oracle_partial* out) {
    int64_t es = elem_size(dtype);
    for (int64_t r = 0; r < B; ++r) {
        oracle_partial p = {0, 0, 0.0, -1};
        const char* row = (const char*)logits + r * row_stride * es;
        const uint32_t* m = mask + r * mask_stride;
        for (int64_t i = 0; i < Vs; ++i) {
            if (!mask_bit(m, i)) continue;
            double v = load_as_double(row, dtype, i);
            if (isnan(v)) { p.nan = 1; continue; }
            if (!p.found || v > p.best) { p.best = v; p.idx = col_offset + i; p.found = 1; }
        }
        out[r] = p;
    }
    return 0;
}

/* parts: [n_shards][B], shards ordered by increasing col_offset */
int oracle_vocab_combine(const oracle_partial* parts, int64_t n_shards, int64_t B,
                         int32_t* out_idx, uint32_t* out_status) {
    for (int64_t r = 0; r < B; ++r) {
        int found = 0, nan = 0;
        double best = 0.0;
        int64_t idx = -1;
        for (int64_t s = 0; s < n_shards; ++s) {
            const oracle_partial* p = &parts[s * B + r];
            nan |= p->nan;
            if (p->found && (!found || p->best > best)) { best = p->best; idx = p->idx; found = 1; }
        }
        if (nan) { out_idx[r] = -1; out_status[r] = OR_NAN_IN_SUPPORT; }
        else if (!found) { out_idx[r] = -1; out_status[r] = OR_EMPTY_MASK; }
        else { out_idx[r] = (int32_t)idx; out_status[r] = (best == -INFINITY) ? OR_ALL_NEG_INF : 0u; }
    }
    return 0;
}

/*
 * Valid-token scan of a dense byte DFA (restating
 * onyx_cuda/rust/src/regex_runtime.rs:129-145 and :197-201): a non-empty token
 * is valid iff walking its bytes from `state` does not end in the dead state.
 * `trans` is [n_states][256]; tokens are CSR (bytes, offsets[V+1]).
 * Writes the packed bitmask (W = ceil(V/32) words, zero tail) for that state.
 */
int oracle_dfa_scan(const int32_t* trans, int32_t n_states, int32_t dead, int32_t state,
                    const uint8_t* tok_bytes, const int64_t* tok_offsets, int64_t V,
                    uint32_t* out_mask) {
    if (state < 0 || state >= n_states) return 1;
    int64_t W = (V + 31) / 32;
    memset(out_mask, 0, (size_t)W * 4);
    for (int64_t t = 0; t < V; ++t) {
        int64_t a = tok_offsets[t], e = tok_offsets[t + 1];
        if (a == e) continue;
        int32_t s = state;
        for (int64_t k = a; k < e; ++k) s = trans[(int64_t)s * 256 + tok_bytes[k]];
        if (s != dead) out_mask[t >> 5] |= 1u << (t & 31);
    }
    return 0;
}

/* one mask row per DFA state: out[s] = oracle_dfa_scan(s) */
int oracle_dfa_table(const int32_t* trans, int32_t n_states, int32_t dead,
                     const uint8_t* tok_bytes, const int64_t* tok_offsets, int64_t V,
                     uint32_t* out_table, int nthreads) {
    set_threads(nthreads);
    int64_t W = (V + 31) / 32;
#pragma omp parallel for schedule(dynamic, 1)
    for (int32_t s = 0; s < n_states; ++s)
        oracle_dfa_scan(trans, n_states, dead, s, tok_bytes, tok_offsets, V, out_table + s * W);
    return 0;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
