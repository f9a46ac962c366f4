// Grammar-masked greedy selection kernels for sm_100a.
//
// One kernel family covers the hot path of bayareahomelander/Onyx's constrained decoding:
//   * masked argmax over logits[rows, vocab] with a packed uint32 valid-token bitmask
//     (replaces TorchCUDAGrammarLogitMask.apply + select_cuda_argmax,
//      onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:69-186, torch_backend.py:970-1007);
//   * the same with each row's mask gathered from a per-DFA-state table by state id;
//   * grammar-aware speculative verify over gamma+1 target rows per batch entry
//     (replaces the per-position loop of grammar_acceptance.py:196-283 and the bonus
//      selection of grammar_continuation.py:127-152);
//   * vocabulary-sharded partial selection emitting packed (order, index) keys, plus the
//     combine of gathered keys.
//
// Work decomposition. Each row is cut into fixed segments; one CTA owns one segment and
// holds all of it in registers (UNROLL 16-byte vectors per thread), so a segment is read
// from HBM exactly once:
//   phase 1  masked, NaN-propagating maximum with packed bf16x2/f16x2 (or f32) max
//            instructions -- no index bookkeeping on the streaming path;
//   phase 2  the thread(s) whose maximum equals the CTA maximum search their registers for
//            the first valid element with that value; the CTA takes the lowest such index.
// Segments of one row (or of one verify batch entry) are merged by the last CTA to finish:
// every CTA stores its 16-byte partial in the caller's workspace, fences, and takes a ticket
// with one atomicAdd; the CTA that draws the final ticket combines the partials, writes the
// outputs and resets the counter to zero for the next call. Nothing ever waits on another
// CTA, so no schedule can hang.
#include "onyx_common.cuh"
#include "../../include/onyx_b200.h"

#include <algorithm>
#include <cstdlib>

namespace onyx {

enum Mode : int { kModeArgmax = 0, kModeKey = 1, kModeVerify = 2 };

struct ScanParams {
  const void* logits;
  int64_t group_stride;  // elements between groups (batch entries)
  int64_t row_stride;    // elements between rows of one group
  int64_t vocab;         // columns scanned per row
  const uint32_t* mask;  // nullptr: every column valid
  int64_t mask_group_stride;  // words
  int64_t mask_row_stride;    // words
  const int32_t* state_ids;   // gather: mask row = mask + state_ids[row] * mask_row_stride
  int64_t n_states;
  int64_t idx_offset;  // global index of column 0 (vocabulary shards)
  int64_t rows;        // total rows = groups * per_group
  int per_group;       // rows per group (gamma + 1 for verify, else 1)
  int segs;            // segments per row
  int64_t seg_elems;   // elements per segment (multiple of 32)
  Partial* ws_part;    // [rows * segs]
  uint32_t* ws_count;  // [groups]
  // outputs
  int32_t* out_idx;
  uint32_t* out_status;
  unsigned long long* out_key;
  // verify
  const int32_t* drafts;
  int64_t draft_stride;
  int bonus;
  int32_t* accept_len;
  int32_t* correction;
};

constexpr int kMaxPerGroup = 256;

template <int THREADS>
__device__ __forceinline__ uint32_t cta_max_u32(uint32_t v, uint32_t* scratch) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < THREADS / 32 ? scratch[lane] : 0u;
    w = __reduce_max_sync(0xFFFFFFFFu, w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  uint32_t r = scratch[32];
  __syncthreads();
  return r;
}

template <int THREADS>
__device__ __forceinline__ uint32_t cta_min_u32(uint32_t v, uint32_t* scratch) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < THREADS / 32 ? scratch[lane] : 0xFFFFFFFFu;
    w = __reduce_min_sync(0xFFFFFFFFu, w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  uint32_t r = scratch[32];
  __syncthreads();
  return r;
}

template <int THREADS>
__device__ __forceinline__ unsigned long long cta_max_u64(unsigned long long v,
                                                          unsigned long long* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = other > v ? other : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = lane < THREADS / 32 ? scratch[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, w, o);
      w = other > w ? other : w;
    }
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  unsigned long long r = scratch[32];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------------------
// fast path: 16-byte aligned rows of bf16 / f16 / f32
// ---------------------------------------------------------------------------------------
template <int DT>
struct Vec16;

// bf16 / f16: 8 elements per vector, packed two per register
template <int DT>
struct Packed16 {
  static constexpr int kElems = 8;
  static constexpr uint32_t kNegInfPair = (DT == kBF16) ? 0xFF80FF80u : 0xFC00FC00u;
  __device__ static uint32_t pmax(uint32_t a, uint32_t b) {
    return DT == kBF16 ? max_nan_bf16x2(a, b) : max_nan_f16x2(a, b);
  }
  __device__ static float half_to_f32(uint32_t h) {
    return DT == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
  }
  // masked maximum of one vector (8 mask bits in `bits`), as a float; -inf if no bit set
  __device__ static uint32_t masked_pair_max(const uint4& x, uint32_t bits) {
    uint32_t m01, m23, m45, m67;
    expand4_16(bits, m01, m23);
    expand4_16(bits >> 4, m45, m67);
    const uint32_t a0 = (x.x & m01) | (kNegInfPair & ~m01);
    const uint32_t a1 = (x.y & m23) | (kNegInfPair & ~m23);
    const uint32_t a2 = (x.z & m45) | (kNegInfPair & ~m45);
    const uint32_t a3 = (x.w & m67) | (kNegInfPair & ~m67);
    return pmax(pmax(a0, a1), pmax(a2, a3));
  }
  __device__ static float pair_to_f32_max(uint32_t pair) {
    return max_nan_f32(half_to_f32(pair & 0xFFFFu), half_to_f32(pair >> 16));
  }
  __device__ static float elem(const uint4& x, int j) {
    const uint32_t w = (j < 2) ? x.x : (j < 4) ? x.y : (j < 6) ? x.z : x.w;
    return half_to_f32((j & 1) ? (w >> 16) : (w & 0xFFFFu));
  }
};

template <>
struct Vec16<kBF16> : Packed16<kBF16> {};
template <>
struct Vec16<kF16> : Packed16<kF16> {};

// f32: 4 elements per vector
template <>
struct Vec16<kF32> {
  static constexpr int kElems = 4;
  __device__ static float masked_max(const uint4& x, uint32_t bits) {
    const float n = __int_as_float(0xFF800000);
    const float a0 = (bits & 1u) ? __uint_as_float(x.x) : n;
    const float a1 = (bits & 2u) ? __uint_as_float(x.y) : n;
    const float a2 = (bits & 4u) ? __uint_as_float(x.z) : n;
    const float a3 = (bits & 8u) ? __uint_as_float(x.w) : n;
    return max_nan_f32(max_nan_f32(a0, a1), max_nan_f32(a2, a3));
  }
  __device__ static float elem(const uint4& x, int j) {
    const uint32_t w = (j == 0) ? x.x : (j == 1) ? x.y : (j == 2) ? x.z : x.w;
    return __uint_as_float(w);
  }
};

template <int DT, int THREADS, int UNROLL>
__device__ __forceinline__ Partial scan_segment_fast(const void* row_base, const uint32_t* mrow,
                                                     int64_t e0, int64_t e1,
                                                     uint32_t* scratch32) {
  using V = Vec16<DT>;
  constexpr int E = V::kElems;
  const int tid = threadIdx.x;
  const int64_t nv = (e1 - e0) / E;  // full vectors in this segment
  const int tail = (int)((e1 - e0) - nv * E);
  const char* rowc = static_cast<const char*>(row_base);
  constexpr int kBytesPerElem = (DT == kF32) ? 4 : 2;

  uint4 x[UNROLL];
  uint32_t bits[UNROLL];
#pragma unroll
  for (int k = 0; k < UNROLL; ++k) {
    const int64_t v = (int64_t)k * THREADS + tid;
    if (v < nv) {
      const int64_t e = e0 + v * E;
      x[k] = ld_stream_v4(rowc + e * kBytesPerElem);
      bits[k] = mrow ? (ld_mask_word(mrow + (e >> 5)) >> (e & 31)) : 0xFFFFFFFFu;
    } else {
      x[k] = make_uint4(0u, 0u, 0u, 0u);
      bits[k] = 0u;
    }
  }
  // ragged end of the row (vocab not a multiple of the vector width): one scalar element
  // per thread, at the highest indices of the segment
  uint32_t tail_raw = 0u, tail_bit = 0u;
  int64_t tail_e = 0;
  if (tid < tail) {
    tail_e = e0 + nv * E + tid;
    if (DT == kF32) {
      tail_raw = __float_as_uint(reinterpret_cast<const float*>(rowc)[tail_e]);
    } else {
      tail_raw = reinterpret_cast<const uint16_t*>(rowc)[tail_e];
    }
    tail_bit = mrow ? ((ld_mask_word(mrow + (tail_e >> 5)) >> (tail_e & 31)) & 1u) : 1u;
  }

  // phase 1: masked maximum, no indices
  constexpr uint32_t kLaneBits = (E == 8) ? 0xFFu : 0xFu;
  uint32_t any = tail_bit;
  float tmax;
  if constexpr (DT == kF32) {
    tmax = __int_as_float(0xFF800000);
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      any |= bits[k] & kLaneBits;
      tmax = max_nan_f32(tmax, V::masked_max(x[k], bits[k]));
    }
    if (tail_bit) tmax = max_nan_f32(tmax, __uint_as_float(tail_raw));
  } else {
    uint32_t pm = V::kNegInfPair;
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      any |= bits[k] & kLaneBits;
      pm = V::pmax(pm, V::masked_pair_max(x[k], bits[k]));
    }
    tmax = V::pair_to_f32_max(pm);
    if (tail_bit) tmax = max_nan_f32(tmax, V::half_to_f32(tail_raw));
  }
  const uint32_t tord = ord32(tmax);
  const int cta_any = __syncthreads_or(any != 0u);
  const uint32_t M = cta_max_u32<THREADS>(tord, scratch32);

  Partial part;
  part.flags = cta_any ? kFlagAny : 0u;
  part.ord = cta_any ? (unsigned long long)M : 0ull;
  part.idx = 0xFFFFFFFFu;
  if (!cta_any || M == kOrd32NaN) return part;

  // phase 2: first valid element equal to the CTA maximum
  uint32_t cand = 0xFFFFFFFFu;
  if (any && tord == M) {
    bool done = false;
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      if (done) break;
      const uint32_t b = bits[k] & kLaneBits;
      if (!b) continue;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        if (!done && ((b >> j) & 1u) && ord32(V::elem(x[k], j)) == M) {
          cand = (uint32_t)(e0 + ((int64_t)k * THREADS + tid) * E + j);
          done = true;
        }
      }
    }
    if (!done && tail_bit) {
      const float tv = (DT == kF32) ? __uint_as_float(tail_raw)
                                    : Packed16<DT == kF32 ? kBF16 : DT>::half_to_f32(tail_raw);
      if (ord32(tv) == M) cand = (uint32_t)tail_e;
    }
  }
  part.idx = cta_min_u32<THREADS>(cand, scratch32);
  return part;
}

// ---------------------------------------------------------------------------------------
// generic path: any alignment, and f64. Scalar coalesced loads; phase 2 re-reads the
// segment (it is still in L2).
// ---------------------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ double load_elem(const void* base, int64_t i) {
  if constexpr (DT == kF64) {
    return __ldg(static_cast<const double*>(base) + i);
  } else if constexpr (DT == kF32) {
    return (double)__ldg(static_cast<const float*>(base) + i);
  } else if constexpr (DT == kBF16) {
    return (double)bf16_bits_to_f32(__ldg(static_cast<const unsigned short*>(base) + i));
  } else {
    return (double)f16_bits_to_f32(__ldg(static_cast<const unsigned short*>(base) + i));
  }
}

template <int DT>
__device__ __forceinline__ unsigned long long elem_ord(double v) {
  if constexpr (DT == kF64) {
    return ord64(v);
  } else {
    return (unsigned long long)ord32((float)v);
  }
}

template <int DT, int THREADS>
__device__ __forceinline__ Partial scan_segment_generic(const void* row_base,
                                                        const uint32_t* mrow, int64_t e0,
                                                        int64_t e1,
                                                        unsigned long long* scratch64) {
  const int tid = threadIdx.x;
  unsigned long long tbest = 0ull;
  uint32_t any = 0u;
  for (int64_t e = e0 + tid; e < e1; e += THREADS) {
    const uint32_t bit = mrow ? ((__ldg(mrow + (e >> 5)) >> (e & 31)) & 1u) : 1u;
    if (bit) {
      any = 1u;
      const unsigned long long o = elem_ord<DT>(load_elem<DT>(row_base, e));
      tbest = o > tbest ? o : tbest;
    }
  }
  const int cta_any = __syncthreads_or(any != 0u);
  const unsigned long long M = cta_max_u64<THREADS>(tbest, scratch64);
  const unsigned long long nan_code = (DT == kF64) ? kOrd64NaN : (unsigned long long)kOrd32NaN;
  Partial part;
  part.flags = cta_any ? kFlagAny : 0u;
  part.ord = cta_any ? M : 0ull;
  part.idx = 0xFFFFFFFFu;
  if (!cta_any || M == nan_code) return part;
  uint32_t cand = 0xFFFFFFFFu;
  if (any && tbest == M) {
    for (int64_t e = e0 + tid; e < e1; e += THREADS) {
      const uint32_t bit = mrow ? ((__ldg(mrow + (e >> 5)) >> (e & 31)) & 1u) : 1u;
      if (bit && elem_ord<DT>(load_elem<DT>(row_base, e)) == M) {
        cand = (uint32_t)e;
        break;
      }
    }
  }
  part.idx = cta_min_u32<THREADS>(cand, reinterpret_cast<uint32_t*>(scratch64));
  return part;
}

// ---------------------------------------------------------------------------------------
// combine + outputs
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void merge(Partial& a, const Partial& b) {
  a.flags |= b.flags & (kFlagBadState | kFlagAboveNegInf);
  if (b.flags & kFlagAny) {
    if (!(a.flags & kFlagAny) || better(b.ord, b.idx, a.ord, a.idx)) {
      a.ord = b.ord;
      a.idx = b.idx;
    }
    a.flags |= kFlagAny;
  }
}

__device__ __forceinline__ Partial empty_partial() {
  Partial p;
  p.ord = 0ull;
  p.idx = 0xFFFFFFFFu;
  p.flags = 0u;
  return p;
}

__device__ __forceinline__ Partial ld_partial_cg(const Partial* p) {
  Partial r;
  const ulonglong2 v = __ldcg(reinterpret_cast<const ulonglong2*>(p));
  r.ord = v.x;
  r.idx = (uint32_t)(v.y & 0xFFFFFFFFull);
  r.flags = (uint32_t)(v.y >> 32);
  return r;
}

__device__ __forceinline__ void st_partial(Partial* p, const Partial& v) {
  ulonglong2 w;
  w.x = v.ord;
  w.y = (unsigned long long)v.idx | ((unsigned long long)v.flags << 32);
  *reinterpret_cast<ulonglong2*>(p) = w;
}

template <int MODE, bool IS64>
__device__ void finalize_group(const ScanParams& p, int64_t group, const Partial* single,
                               Partial* res /* smem [per_group] */) {
  const int P = p.per_group;
  if (single) {
    if (threadIdx.x == 0) res[0] = *single;
  } else {
    // one warp per member row: reduce its `segs` partials
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const Partial* base = p.ws_part + group * (int64_t)P * p.segs;
    for (int i = warp; i < P; i += nwarps) {
      Partial acc = empty_partial();
      for (int s = lane; s < p.segs; s += 32) {
        Partial* slot = const_cast<Partial*>(base) + (int64_t)i * p.segs + s;
        merge(acc, ld_partial_cg(slot));
        // leave the workspace zero-filled: the next call may lay it out differently
        __stcg(reinterpret_cast<ulonglong2*>(slot), make_ulonglong2(0ull, 0ull));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        Partial other;
        other.ord = __shfl_xor_sync(0xFFFFFFFFu, acc.ord, o);
        other.idx = __shfl_xor_sync(0xFFFFFFFFu, acc.idx, o);
        other.flags = __shfl_xor_sync(0xFFFFFFFFu, acc.flags, o);
        merge(acc, other);
      }
      if (lane == 0) res[i] = acc;
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;

  if constexpr (MODE == kModeArgmax) {
    decode_partial(res[0], IS64, &p.out_idx[group], &p.out_status[group]);
  } else if constexpr (MODE == kModeKey) {
    const Partial& r = res[0];
    unsigned long long key = 0ull;
    if (r.flags & kFlagAny) key = (r.ord << 32) | (unsigned long long)(0xFFFFFFFFu - r.idx);
    p.out_key[group] = key;
  } else {
    const int G = P - 1;
    int32_t acc = G, corr = -1;
    uint32_t st = 0u;
    bool decided = false;
    for (int i = 0; i < G && !decided; ++i) {
      int32_t sel;
      uint32_t rs;
      decode_partial(res[i], IS64, &sel, &rs);
      if (rs) {
        acc = i;
        st = rs;
        decided = true;
      } else if (sel != p.drafts[group * p.draft_stride + i]) {
        acc = i;
        corr = sel;
        decided = true;
      }
    }
    if (!decided && p.bonus) {
      int32_t sel;
      uint32_t rs;
      decode_partial(res[G], IS64, &sel, &rs);
      if (rs) {
        st = rs;
      } else {
        corr = sel;
      }
    }
    p.accept_len[group] = acc;
    p.correction[group] = corr;
    p.out_status[group] = st;
  }
}

template <int DT, bool FAST, int MODE, int THREADS, int UNROLL>
__global__ void __launch_bounds__(THREADS)
    masked_select_kernel(const ScanParams p) {
  __shared__ unsigned long long scratch64[33];
  __shared__ Partial res[(MODE == kModeVerify) ? kMaxPerGroup : 1];
  __shared__ int s_last;
  uint32_t* scratch32 = reinterpret_cast<uint32_t*>(scratch64);

  const int64_t blk = blockIdx.x;
  const int64_t row = blk / p.segs;
  const int seg = (int)(blk - row * p.segs);
  const int64_t group = row / p.per_group;
  const int64_t member = row - group * p.per_group;

  // Programmatic dependent launch: everything this kernel reads may come from the
  // preceding kernel in the stream.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  using St = typename Elem<DT>::storage;
  const St* row_base = static_cast<const St*>(p.logits) + group * p.group_stride +
                       member * p.row_stride;
  const uint32_t* mrow = nullptr;
  bool bad_state = false;
  if (p.mask) {
    if (p.state_ids) {
      const int32_t s = __ldg(p.state_ids + row);
      bad_state = (s < 0) || ((int64_t)s >= p.n_states);
      mrow = p.mask + (bad_state ? 0 : (int64_t)s * p.mask_row_stride);
    } else {
      mrow = p.mask + group * p.mask_group_stride + member * p.mask_row_stride;
    }
  }
  const int64_t e0 = (int64_t)seg * p.seg_elems;
  const int64_t e1 = min(e0 + p.seg_elems, p.vocab);

  Partial part;
  if (bad_state) {
    part = empty_partial();
    part.flags = kFlagBadState;
  } else if constexpr (FAST) {
    part = scan_segment_fast<DT, THREADS, UNROLL>(row_base, mrow, e0, e1, scratch32);
  } else {
    part = scan_segment_generic<DT, THREADS>(row_base, mrow, e0, e1, scratch64);
  }
  if (part.idx != 0xFFFFFFFFu) part.idx += (uint32_t)p.idx_offset;

  // let the next kernel in the stream start its prologue
  asm volatile("griddepcontrol.launch_dependents;" :::);

  const int total = p.per_group * p.segs;
  if (total == 1) {
    finalize_group<MODE, DT == kF64>(p, group, &part, res);
    return;
  }
  if (threadIdx.x == 0) {
    st_partial(p.ws_part + blk, part);
    __threadfence();
    const uint32_t t = atomicAdd(p.ws_count + group, 1u);
    s_last = (t == (uint32_t)(total - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  finalize_group<MODE, DT == kF64>(p, group, nullptr, res);
  if (threadIdx.x == 0) p.ws_count[group] = 0u;  // ready for the next call
}

// ---------------------------------------------------------------------------------------
// mask apply: out = allowed values bit-for-bit, -inf elsewhere; per-row status for the
// reference's rejections (empty support, all -inf support; torch_grammar_mask.py:182-185)
// ---------------------------------------------------------------------------------------
struct ApplyParams {
  const void* in;
  int64_t in_stride;
  void* out;
  int64_t out_stride;
  int64_t vocab;
  const uint32_t* mask;
  int64_t mask_stride;
  int64_t rows;
  int segs;
  int64_t seg_elems;
  uint32_t* ws_flags;  // [rows] OR-accumulated flags
  uint32_t* ws_count;  // [rows]
  uint32_t* out_status;
};

__device__ __forceinline__ void st_stream_v4(void* p, const uint4& v) {
  asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

template <int DT>
__device__ __forceinline__ uint4 apply_vec(const uint4& x, uint32_t bits, uint32_t& above) {
  uint4 o;
  if constexpr (DT == kBF16 || DT == kF16) {
    constexpr uint32_t n = (DT == kBF16) ? 0xFF80FF80u : 0xFC00FC00u;
    uint32_t m01, m23, m45, m67;
    expand4_16(bits, m01, m23);
    expand4_16(bits >> 4, m45, m67);
    o.x = (x.x & m01) | (n & ~m01);
    o.y = (x.y & m23) | (n & ~m23);
    o.z = (x.z & m45) | (n & ~m45);
    o.w = (x.w & m67) | (n & ~m67);
    above |= (o.x != n) | (o.y != n) | (o.z != n) | (o.w != n);
  } else if constexpr (DT == kF32) {
    constexpr uint32_t n = 0xFF800000u;
    o.x = (bits & 1u) ? x.x : n;
    o.y = (bits & 2u) ? x.y : n;
    o.z = (bits & 4u) ? x.z : n;
    o.w = (bits & 8u) ? x.w : n;
    above |= (o.x != n) | (o.y != n) | (o.z != n) | (o.w != n);
  } else {  // f64: two elements
    constexpr uint32_t nhi = 0xFFF00000u;
    o.x = (bits & 1u) ? x.x : 0u;
    o.y = (bits & 1u) ? x.y : nhi;
    o.z = (bits & 2u) ? x.z : 0u;
    o.w = (bits & 2u) ? x.w : nhi;
    above |= (o.x != 0u) | (o.y != nhi) | (o.z != 0u) | (o.w != nhi);
  }
  return o;
}

template <int DT>
__device__ __forceinline__ void apply_scalar(const void* in, void* out, int64_t e, uint32_t bit,
                                             uint32_t& above) {
  if constexpr (DT == kBF16 || DT == kF16) {
    const uint16_t n = (DT == kBF16) ? 0xFF80u : 0xFC00u;
    const uint16_t v = bit ? static_cast<const uint16_t*>(in)[e] : n;
    static_cast<uint16_t*>(out)[e] = v;
    above |= (v != n);
  } else if constexpr (DT == kF32) {
    const uint32_t n = 0xFF800000u;
    const uint32_t v = bit ? static_cast<const uint32_t*>(in)[e] : n;
    static_cast<uint32_t*>(out)[e] = v;
    above |= (v != n);
  } else {
    const unsigned long long n = 0xFFF0000000000000ull;
    const unsigned long long v = bit ? static_cast<const unsigned long long*>(in)[e] : n;
    static_cast<unsigned long long*>(out)[e] = v;
    above |= (v != n);
  }
}

template <int DT, bool FAST, int THREADS, int UNROLL>
__global__ void __launch_bounds__(THREADS) mask_apply_kernel(const ApplyParams p) {
  __shared__ int s_last;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t blk = blockIdx.x;
  const int64_t row = blk / p.segs;
  const int seg = (int)(blk - row * p.segs);
  constexpr int ES = Elem<DT>::kBytes;
  const char* in = static_cast<const char*>(p.in) + row * p.in_stride * ES;
  char* out = static_cast<char*>(p.out) + row * p.out_stride * ES;
  const uint32_t* mrow = p.mask + row * p.mask_stride;
  const int64_t e0 = (int64_t)seg * p.seg_elems;
  const int64_t e1 = min(e0 + p.seg_elems, p.vocab);
  uint32_t any = 0u, above = 0u;
  if constexpr (FAST) {
    constexpr int E = 16 / ES;
    constexpr uint32_t lane_bits = (1u << E) - 1u;
    const int64_t nv = (e1 - e0) / E;
    for (int64_t v = threadIdx.x; v < nv; v += THREADS) {
      const int64_t e = e0 + v * E;
      const uint4 x = ld_stream_v4(in + e * ES);
      const uint32_t bits = (ld_mask_word(mrow + (e >> 5)) >> (e & 31)) & lane_bits;
      any |= bits;
      st_stream_v4(out + e * ES, apply_vec<DT>(x, bits, above));
    }
    for (int64_t e = e0 + nv * E + threadIdx.x; e < e1; e += THREADS) {
      const uint32_t bit = (__ldg(mrow + (e >> 5)) >> (e & 31)) & 1u;
      any |= bit;
      apply_scalar<DT>(in, out, e, bit, above);
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += THREADS) {
      const uint32_t bit = (__ldg(mrow + (e >> 5)) >> (e & 31)) & 1u;
      any |= bit;
      apply_scalar<DT>(in, out, e, bit, above);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const uint32_t flags = (__syncthreads_or(any != 0u) ? kFlagAny : 0u) |
                         (__syncthreads_or(above != 0u) ? kFlagAboveNegInf : 0u);
  uint32_t total_flags = flags;
  if (p.segs > 1) {
    if (threadIdx.x == 0) {
      if (flags) atomicOr(p.ws_flags + row, flags);
      __threadfence();
      const uint32_t t = atomicAdd(p.ws_count + row, 1u);
      s_last = (t == (uint32_t)(p.segs - 1));
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) {
      total_flags = __ldcg(p.ws_flags + row);
      p.ws_flags[row] = 0u;
      p.ws_count[row] = 0u;
    }
  }
  if (threadIdx.x == 0) {
    p.out_status[row] = !(total_flags & kFlagAny)
                            ? kStatusEmptyMask
                            : ((total_flags & kFlagAboveNegInf) ? 0u : kStatusAllNegInf);
  }
}

// combine gathered vocabulary-shard keys: keys[part * rows + row]
__global__ void combine_keys_kernel(const unsigned long long* keys, int64_t n_parts, int64_t rows,
                                    int32_t* out_idx, uint32_t* out_status) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  unsigned long long best = 0ull;
  for (int64_t s = 0; s < n_parts; ++s) {
    const unsigned long long k = keys[s * rows + r];
    best = k > best ? k : best;
  }
  Partial pr;
  pr.flags = best ? kFlagAny : 0u;
  pr.ord = best >> 32;
  pr.idx = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
  decode_partial(pr, false, &out_idx[r], &out_status[r]);
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
constexpr int kThreads = 256;
constexpr int kUnroll = 8;
constexpr int kGenericPerThread = 16;

static thread_local int g_last_cuda_error = 0;

struct Plan {
  bool fast;
  int64_t seg_elems;
  int segs;
};

static int vec_elems(int dt) { return dt == kF32 ? 4 : 8; }

static Plan make_plan(int dt, int64_t vocab, bool aligned) {
  Plan pl;
  pl.fast = aligned && (dt == kF32 || dt == kF16 || dt == kBF16);
  pl.seg_elems = pl.fast ? (int64_t)kThreads * kUnroll * vec_elems(dt)
                         : (int64_t)kThreads * kGenericPerThread;
  pl.segs = (int)((vocab + pl.seg_elems - 1) / pl.seg_elems);
  return pl;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static size_t workspace_bytes_for(int64_t rows, int64_t groups, const Plan& pl, int per_group) {
  if ((int64_t)pl.segs * per_group == 1) return 0;
  return align_up((size_t)rows * pl.segs * sizeof(Partial), 256) +
         align_up((size_t)groups * sizeof(uint32_t), 256);
}

template <int DT, bool FAST, int MODE>
static cudaError_t launch_t(const ScanParams& p, cudaStream_t stream, bool pdl) {
  const int64_t blocks = p.rows * p.segs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, masked_select_kernel<DT, FAST, MODE, kThreads, kUnroll>, p);
}

template <int MODE>
static cudaError_t dispatch(int dt, bool fast, const ScanParams& p, cudaStream_t s, bool pdl) {
  switch (dt) {
    case kBF16:
      return fast ? launch_t<kBF16, true, MODE>(p, s, pdl) : launch_t<kBF16, false, MODE>(p, s, pdl);
    case kF16:
      return fast ? launch_t<kF16, true, MODE>(p, s, pdl) : launch_t<kF16, false, MODE>(p, s, pdl);
    case kF32:
      return fast ? launch_t<kF32, true, MODE>(p, s, pdl) : launch_t<kF32, false, MODE>(p, s, pdl);
    case kF64:
      if constexpr (MODE == kModeKey) return cudaErrorInvalidValue;
      return launch_t<kF64, false, MODE>(p, s, pdl);
  }
  return cudaErrorInvalidValue;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static int finish_launch(cudaError_t e) {
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  return ONYX_OK;
}

static bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("ONYX_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

static int bind_workspace(ScanParams& p, void* ws, size_t ws_bytes, size_t need,
                          int64_t groups) {
  if (need == 0) {
    p.ws_part = nullptr;
    p.ws_count = nullptr;
    return ONYX_OK;
  }
  if (!ws || ws_bytes < need || ((uintptr_t)ws & 255u)) return ONYX_ERR_WORKSPACE;
  const size_t part_bytes = align_up((size_t)p.rows * p.segs * sizeof(Partial), 256);
  p.ws_part = static_cast<Partial*>(ws);
  p.ws_count = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + part_bytes);
  (void)groups;
  return ONYX_OK;
}

static bool dtype_ok(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16 || dt == kF64; }

}  // namespace onyx

using namespace onyx;

extern "C" {

int onyx_abi_version(void) { return ONYX_ABI_VERSION; }

int onyx_last_cuda_error(void) { return g_last_cuda_error; }

const char* onyx_error_string(int code) {
  switch (code) {
    case ONYX_OK: return "ok";
    case ONYX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ONYX_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case ONYX_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case ONYX_ERR_CUDA: return "CUDA launch failed (see onyx_last_cuda_error)";
  }
  return "unknown error";
}

size_t onyx_masked_argmax_workspace_size(int64_t rows, int64_t vocab, int dtype) {
  if (rows <= 0 || vocab <= 0 || !dtype_ok(dtype)) return 0;
  // worst case over alignments: the generic plan has the most segments
  const Plan a = make_plan(dtype, vocab, true), b = make_plan(dtype, vocab, false);
  return std::max(workspace_bytes_for(rows, rows, a, 1), workspace_bytes_for(rows, rows, b, 1));
}

size_t onyx_spec_verify_workspace_size(int64_t batch, int64_t gamma, int64_t vocab, int dtype) {
  if (batch <= 0 || gamma < 1 || vocab <= 0 || !dtype_ok(dtype)) return 0;
  const int64_t rows = batch * (gamma + 1);
  const Plan a = make_plan(dtype, vocab, true), b = make_plan(dtype, vocab, false);
  return std::max(workspace_bytes_for(rows, batch, a, (int)(gamma + 1)),
                  workspace_bytes_for(rows, batch, b, (int)(gamma + 1)));
}

static int common_checks(const void* logits, int dtype, int64_t rows, int64_t vocab,
                         int64_t row_stride) {
  if (!dtype_ok(dtype)) return ONYX_ERR_UNSUPPORTED_DTYPE;
  if (rows < 0 || vocab <= 0 || vocab > 0x7FFFFFFFll - 1) return ONYX_ERR_INVALID_ARGUMENT;
  if (rows > 0 && !logits) return ONYX_ERR_INVALID_ARGUMENT;
  if (row_stride < vocab && rows > 1) return ONYX_ERR_INVALID_ARGUMENT;
  return ONYX_OK;
}

int onyx_masked_argmax(const void* logits, int dtype, int64_t rows, int64_t vocab,
                       int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                       int32_t* out_idx, uint32_t* out_status, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = common_checks(logits, dtype, rows, vocab, row_stride);
  if (rc) return rc;
  if (rows == 0) return ONYX_OK;
  if (!out_idx || !out_status) return ONYX_ERR_INVALID_ARGUMENT;
  if (mask && mask_stride < (vocab + 31) / 32 && rows > 1) return ONYX_ERR_INVALID_ARGUMENT;
  const int es = dtype_bytes(dtype);
  const bool aligned = aligned16(logits) && ((row_stride * es) % 16 == 0 || rows == 1);
  const Plan pl = make_plan(dtype, vocab, aligned);
  ScanParams p = {};
  p.logits = logits;
  p.group_stride = row_stride;
  p.row_stride = 0;
  p.vocab = vocab;
  p.mask = mask;
  p.mask_group_stride = mask_stride;
  p.mask_row_stride = 0;
  p.rows = rows;
  p.per_group = 1;
  p.segs = pl.segs;
  p.seg_elems = pl.seg_elems;
  p.out_idx = out_idx;
  p.out_status = out_status;
  rc = bind_workspace(p, workspace, workspace_bytes, workspace_bytes_for(rows, rows, pl, 1), rows);
  if (rc) return rc;
  return finish_launch(dispatch<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}

int onyx_gather_masked_argmax(const void* logits, int dtype, int64_t rows, int64_t vocab,
                              int64_t row_stride, const uint32_t* table, int64_t n_states,
                              int64_t table_stride, const int32_t* state_ids, int32_t* out_idx,
                              uint32_t* out_status, void* workspace, size_t workspace_bytes,
                              void* stream) {
  int rc = common_checks(logits, dtype, rows, vocab, row_stride);
  if (rc) return rc;
  if (rows == 0) return ONYX_OK;
  if (!table || !state_ids || !out_idx || !out_status || n_states <= 0)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (table_stride < (vocab + 31) / 32) return ONYX_ERR_INVALID_ARGUMENT;
  const int es = dtype_bytes(dtype);
  const bool aligned = aligned16(logits) && ((row_stride * es) % 16 == 0 || rows == 1);
  const Plan pl = make_plan(dtype, vocab, aligned);
  ScanParams p = {};
  p.logits = logits;
  p.group_stride = row_stride;
  p.vocab = vocab;
  p.mask = table;
  p.mask_row_stride = table_stride;
  p.state_ids = state_ids;
  p.n_states = n_states;
  p.rows = rows;
  p.per_group = 1;
  p.segs = pl.segs;
  p.seg_elems = pl.seg_elems;
  p.out_idx = out_idx;
  p.out_status = out_status;
  rc = bind_workspace(p, workspace, workspace_bytes, workspace_bytes_for(rows, rows, pl, 1), rows);
  if (rc) return rc;
  return finish_launch(dispatch<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}

int onyx_spec_verify(const void* logits, int dtype, int64_t batch, int64_t gamma, int64_t vocab,
                     int64_t batch_stride, int64_t row_stride, const uint32_t* masks,
                     int64_t mask_batch_stride, int64_t mask_row_stride, const int32_t* drafts,
                     int64_t draft_stride, int bonus, int32_t* accept_len, int32_t* correction,
                     uint32_t* out_status, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (!dtype_ok(dtype)) return ONYX_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || gamma < 1 || gamma + 1 > kMaxPerGroup || vocab <= 0 ||
      vocab > 0x7FFFFFFFll - 1)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (batch == 0) return ONYX_OK;
  if (!logits || !masks || !drafts || !accept_len || !correction || !out_status)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (row_stride < vocab || mask_row_stride < (vocab + 31) / 32) return ONYX_ERR_INVALID_ARGUMENT;
  if (batch > 1 && (batch_stride < (gamma + 1) * row_stride ||
                    mask_batch_stride < (gamma + 1) * mask_row_stride || draft_stride < gamma))
    return ONYX_ERR_INVALID_ARGUMENT;
  const int es = dtype_bytes(dtype);
  const bool aligned = aligned16(logits) && (row_stride * es) % 16 == 0 &&
                       ((batch_stride * es) % 16 == 0 || batch == 1);
  const Plan pl = make_plan(dtype, vocab, aligned);
  const int P = (int)(gamma + 1);
  ScanParams p = {};
  p.logits = logits;
  p.group_stride = batch_stride;
  p.row_stride = row_stride;
  p.vocab = vocab;
  p.mask = masks;
  p.mask_group_stride = mask_batch_stride;
  p.mask_row_stride = mask_row_stride;
  p.rows = batch * P;
  p.per_group = P;
  p.segs = pl.segs;
  p.seg_elems = pl.seg_elems;
  p.out_status = out_status;
  p.drafts = drafts;
  p.draft_stride = draft_stride;
  p.bonus = bonus ? 1 : 0;
  p.accept_len = accept_len;
  p.correction = correction;
  const int rc = bind_workspace(p, workspace, workspace_bytes,
                                workspace_bytes_for(p.rows, batch, pl, P), batch);
  if (rc) return rc;
  return finish_launch(dispatch<kModeVerify>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}

size_t onyx_vocab_partial_workspace_size(int64_t rows, int64_t shard_vocab, int dtype) {
  if (dtype == kF64) return 0;
  return onyx_masked_argmax_workspace_size(rows, shard_vocab, dtype);
}

int onyx_vocab_partial_argmax(const void* logits, int dtype, int64_t rows, int64_t shard_vocab,
                              int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                              int64_t col_offset, uint64_t* out_keys, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (dtype == kF64) return ONYX_ERR_UNSUPPORTED_DTYPE;
  int rc = common_checks(logits, dtype, rows, shard_vocab, row_stride);
  if (rc) return rc;
  if (rows == 0) return ONYX_OK;
  if (!mask || !out_keys || col_offset < 0 || (col_offset & 31) ||
      col_offset + shard_vocab > 0x7FFFFFFFll - 1)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (mask_stride < (shard_vocab + 31) / 32 && rows > 1) return ONYX_ERR_INVALID_ARGUMENT;
  const int es = dtype_bytes(dtype);
  const bool aligned = aligned16(logits) && ((row_stride * es) % 16 == 0 || rows == 1);
  const Plan pl = make_plan(dtype, shard_vocab, aligned);
  ScanParams p = {};
  p.logits = logits;
  p.group_stride = row_stride;
  p.vocab = shard_vocab;
  p.mask = mask;
  p.mask_group_stride = mask_stride;
  p.idx_offset = col_offset;
  p.rows = rows;
  p.per_group = 1;
  p.segs = pl.segs;
  p.seg_elems = pl.seg_elems;
  p.out_key = reinterpret_cast<unsigned long long*>(out_keys);
  rc = bind_workspace(p, workspace, workspace_bytes, workspace_bytes_for(rows, rows, pl, 1), rows);
  if (rc) return rc;
  return finish_launch(dispatch<kModeKey>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}

static Plan make_apply_plan(int dt, int64_t vocab, bool aligned) {
  Plan pl;
  pl.fast = aligned;
  pl.seg_elems = (int64_t)kThreads * kUnroll * (16 / dtype_bytes(dt));
  pl.segs = (int)((vocab + pl.seg_elems - 1) / pl.seg_elems);
  return pl;
}

size_t onyx_mask_apply_workspace_size(int64_t rows, int64_t vocab, int dtype) {
  if (rows <= 0 || vocab <= 0 || !dtype_ok(dtype)) return 0;
  const Plan pl = make_apply_plan(dtype, vocab, true);
  if (pl.segs == 1) return 0;
  return align_up((size_t)rows * 2 * sizeof(uint32_t), 256);
}

int onyx_mask_apply(const void* logits, int dtype, int64_t rows, int64_t vocab,
                    int64_t row_stride, const uint32_t* mask, int64_t mask_stride, void* out,
                    int64_t out_stride, uint32_t* out_status, void* workspace,
                    size_t workspace_bytes, void* stream) {
  int rc = common_checks(logits, dtype, rows, vocab, row_stride);
  if (rc) return rc;
  if (rows == 0) return ONYX_OK;
  if (!mask || !out || !out_status) return ONYX_ERR_INVALID_ARGUMENT;
  if (rows > 1 && (out_stride < vocab || mask_stride < (vocab + 31) / 32))
    return ONYX_ERR_INVALID_ARGUMENT;
  const int es = dtype_bytes(dtype);
  const bool aligned = aligned16(logits) && aligned16(out) &&
                       (rows == 1 || ((row_stride * es) % 16 == 0 && (out_stride * es) % 16 == 0));
  const Plan pl = make_apply_plan(dtype, vocab, aligned);
  ApplyParams p = {};
  p.in = logits;
  p.in_stride = row_stride;
  p.out = out;
  p.out_stride = out_stride;
  p.vocab = vocab;
  p.mask = mask;
  p.mask_stride = mask_stride;
  p.rows = rows;
  p.segs = pl.segs;
  p.seg_elems = pl.seg_elems;
  p.out_status = out_status;
  if (pl.segs > 1) {
    const size_t need = align_up((size_t)rows * 2 * sizeof(uint32_t), 256);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u))
      return ONYX_ERR_WORKSPACE;
    p.ws_flags = static_cast<uint32_t*>(workspace);
    p.ws_count = p.ws_flags + rows;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * pl.segs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaErrorInvalidValue;
#define ONYX_APPLY_CASE(DTV)                                                                   \
  case DTV:                                                                                    \
    e = pl.fast ? cudaLaunchKernelEx(&cfg, mask_apply_kernel<DTV, true, kThreads, kUnroll>, p) \
                : cudaLaunchKernelEx(&cfg, mask_apply_kernel<DTV, false, kThreads, kUnroll>, p); \
    break;
  switch (dtype) {
    ONYX_APPLY_CASE(kBF16)
    ONYX_APPLY_CASE(kF16)
    ONYX_APPLY_CASE(kF32)
    ONYX_APPLY_CASE(kF64)
  }
#undef ONYX_APPLY_CASE
  return finish_launch(e);
}

int onyx_combine_partials(const uint64_t* keys, int64_t n_parts, int64_t rows, int32_t* out_idx,
                          uint32_t* out_status, void* stream) {
  if (n_parts <= 0 || rows < 0) return ONYX_ERR_INVALID_ARGUMENT;
  if (rows == 0) return ONYX_OK;
  if (!keys || !out_idx || !out_status) return ONYX_ERR_INVALID_ARGUMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rows + 255) / 256), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return finish_launch(cudaLaunchKernelEx(&cfg, combine_keys_kernel,
                                          reinterpret_cast<const unsigned long long*>(keys),
                                          n_parts, rows, out_idx, out_status));
}

}  // extern "C"
