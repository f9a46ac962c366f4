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

#include <cuda.h>  // CUcontext / CUresult only: the driver entry point is looked up at run time


#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#ifndef ONYX_PDL_EARLY
#define ONYX_PDL_EARLY 0
#endif

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
  int segs;            // warp segments per row
  int ctas_per_row;    // CTAs per row (each covers blockDim/32 consecutive segments)
  int64_t seg_elems;   // elements per warp segment (multiple of 32)
  Partial* ws_part;    // [rows * ctas_per_row], one partial per CTA
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
  // test hook: key bytes rank 0 of the cluster path expects beyond those sent (0 normally;
  // nonzero makes its bounded wait run out)
  uint32_t withheld_key_bytes;
  // key mode with a peer exchange: row r's key goes to key_dst[i][parity * key_parity_stride
  // + r] for every i < n_key_dst (this rank's slot in every rank's exchange buffer, the
  // peers' over NVLink) instead of out_key; the parity is that of this call's epoch, one
  // above the count kept in this rank's buffer at key_epoch
  unsigned long long* key_dst[8];
  int n_key_dst;
  int64_t key_parity_stride;
  const unsigned long long* key_epoch;
  const unsigned long long* key_failed;  // nonzero: the exchange failed, store no key
};

constexpr int kMaxPerGroup = 256;
constexpr uint32_t kFull = 0xFFFFFFFFu;

// ---------------------------------------------------------------------------------------
// fast path: 16-byte aligned rows of bf16 / f16 / f32. One warp owns one segment of
// 32 lanes x UNROLL vectors; every load of the segment is issued before any is consumed.
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
  // masked maximum of one vector (8 mask bits in `bits`), as a packed pair
  __device__ static uint32_t masked_pair_max(const uint4& x, uint32_t bits) {
    uint32_t m01, m23, m45, m67;
    expand8_16(bits, m01, m23, m45, m67);
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
  __device__ static float scalar(uint32_t raw) { return half_to_f32(raw); }
  // the 16-bit pattern of a float that came from this type (exact)
  __device__ static uint32_t from_f32(float f) {
    if constexpr (DT == kBF16) {
      return __float_as_uint(f) >> 16;
    } else {
      return __half_as_ushort(__float2half_rn(f));
    }
  }
  // 0xFFFF in each 16-bit lane of a equal (as floats) to the same lane of b
  __device__ static uint32_t eq_mask(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (DT == kBF16) {
      asm("set.eq.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    } else {
      asm("set.eq.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    }
    return d;
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
  __device__ static float scalar(uint32_t raw) { return __uint_as_float(raw); }
};

// One warp's segment [e0, e1) of a row, held in registers: 32 lanes x UNROLL 16-byte
// vectors, every load issued before any is consumed, plus one ragged-tail element per lane
// when the row length is not a multiple of the vector width.
//   phase 1 (max_code): masked, NaN-propagating maximum with packed max instructions and no
//            index bookkeeping; each vector's own maximum is kept.
//   phase 2 (first_index): given a value code M, the lowest index holding it -- the first
//            (vector k, lane) whose kept maximum equals M, then the first valid element of
//            that vector equal to M. Element order within the segment is (k, lane, j).
template <int DT, int UNROLL>
struct WarpSegment {
  using V = Vec16<DT>;
  static constexpr int E = V::kElems;
  static constexpr int kBytesPerElem = (DT == kF32) ? 4 : 2;
  static constexpr uint32_t kLaneBits = (E == 8) ? 0xFFu : 0xFu;

  uint4 x[UNROLL];
  uint32_t bits[UNROLL];
  uint32_t tail_raw, tail_bit;
  uint32_t tord;  // this lane's maximum as an order code, 0 = no valid token
  uint32_t vm[(DT == kF32) ? 1 : UNROLL];  // 16-bit types: each vector's masked pair maximum
  uint32_t e0, nv;  // in-row indices are 32-bit: rows are shorter than 2^31 elements
  int lane;

  __device__ __forceinline__ void load(const void* row_base, const uint32_t* mrow, int64_t e0_,
                                       int64_t e1, int lane_) {
    e0 = (uint32_t)e0_;
    lane = lane_;
    const uint32_t n = (uint32_t)(e1 - e0_);
    nv = n / E;  // full vectors in this segment
    const int tail = (int)(n - nv * E);
    const char* rowc = static_cast<const char*>(row_base);
    // the lane's first vector and, in each group of 32 vectors, its mask word: segment
    // starts and vector strides are multiples of 32 elements
    const uint4* vp = reinterpret_cast<const uint4*>(rowc + (size_t)e0 * kBytesPerElem) + lane;
    const uint32_t* mp = mrow ? mrow + (e0 >> 5) + ((lane * E) >> 5) : nullptr;
    uint32_t w[UNROLL];
    if (nv == (uint32_t)(UNROLL * 32)) {  // full segment (warp-uniform): no bounds checks
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        x[k] = __ldcs(vp + k * 32);
        w[k] = mp ? __ldg(mp + k * E) : 0xFFFFFFFFu;
      }
    } else {
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        if ((uint32_t)(k * 32 + lane) < nv) {
          x[k] = __ldcs(vp + k * 32);
          w[k] = mp ? __ldg(mp + k * E) : 0xFFFFFFFFu;
        } else {
          x[k] = make_uint4(0u, 0u, 0u, 0u);
          w[k] = 0u;
        }
      }
    }
    tail_raw = 0u;
    tail_bit = 0u;
    if (lane < tail) {
      const uint32_t te = e0 + nv * E + lane;
      if (DT == kF32) {
        tail_raw = __float_as_uint(__ldg(reinterpret_cast<const float*>(rowc) + te));
      } else {
        tail_raw = __ldg(reinterpret_cast<const unsigned short*>(rowc) + te);
      }
      tail_bit = mrow ? ((__ldg(mrow + (te >> 5)) >> (te & 31)) & 1u) : 1u;
    }
    // the lane's mask bits in the low bits; higher bits (other lanes') are ignored by
    // every consumer
    const uint32_t lane_shift = (uint32_t)(lane * E) & 31u;
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) bits[k] = w[k] >> lane_shift;
  }

  // warp maximum as an order code (0: no valid token in the segment)
  __device__ __forceinline__ uint32_t max_code() {
    uint32_t any = 0u;
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) any |= bits[k];
    any = (any & kLaneBits) | tail_bit;
    float tmax;
    if constexpr (DT == kF32) {
      tmax = __int_as_float(0xFF800000);
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) tmax = max_nan_f32(tmax, V::masked_max(x[k], bits[k]));
    } else {
      uint32_t pm = V::kNegInfPair;
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        vm[k] = V::masked_pair_max(x[k], bits[k]);
        pm = V::pmax(pm, vm[k]);
      }
      tmax = V::pair_to_f32_max(pm);
    }
    if (tail_bit) tmax = max_nan_f32(tmax, V::scalar(tail_raw));
    tord = any ? ord32(tmax) : 0u;
    return __reduce_max_sync(kFull, tord);
  }

  // lowest index of the segment whose valid value has order code M (a code of a real,
  // non-NaN value); 0xFFFFFFFF if the segment holds none. Warp-wide, lanes converged.
  // Equality is float equality, so -0.0 and +0.0 match alike.
  __device__ __forceinline__ uint32_t first_index(uint32_t M) {
    const float mf = __uint_as_float((M & 0x80000000u) ? (M & 0x7FFFFFFFu) : ~M);
    uint32_t key = 0xFFFFFFFFu;
    uint32_t m2 = 0u;
    if constexpr (DT == kF32) {
      if (tord == M) {  // only lanes whose maximum is M can hold it
        // f32 keeps no per-vector maxima: recompute them in the lanes that get here
#pragma unroll
        for (int k = UNROLL - 1; k >= 0; --k)
          if ((bits[k] & kLaneBits) && V::masked_max(x[k], bits[k]) == mf)
            key = ((uint32_t)k << 5) | lane;
      }
    } else {
      // branch-free over the lanes: which kept vector maxima equal M, as a bit per vector
      const uint32_t h = V::from_f32(mf);
      m2 = h | (h << 16);
      uint32_t hit = 0u;
#pragma unroll
      for (int k = 0; k < UNROLL; ++k)
        hit |= ((bits[k] & kLaneBits) && V::eq_mask(vm[k], m2)) ? (1u << k) : 0u;
      if (tord == M && hit) key = ((uint32_t)(__ffs(hit) - 1) << 5) | lane;
    }
    if (tord == M && key == 0xFFFFFFFFu && tail_bit && ord32(V::scalar(tail_raw)) == M)
      key = ((uint32_t)UNROLL << 5) | lane;  // the ragged tail follows every full vector
    const uint32_t win = __reduce_min_sync(kFull, key);
    if (win == 0xFFFFFFFFu) return 0xFFFFFFFFu;
    const int wk = (int)(win >> 5), wl = (int)(win & 31u);
    if (wk >= UNROLL) return e0 + nv * E + (uint32_t)wl;
    uint4 xv = x[0];
    uint32_t bv = bits[0];
#pragma unroll
    for (int k = 1; k < UNROLL; ++k)
      if (k == wk) {  // warp-uniform
        xv = x[k];
        bv = bits[k];
      }
    int j;
    if constexpr (DT == kF32) {
      j = 3;
      if ((bv & 4u) && __uint_as_float(xv.z) == mf) j = 2;
      if ((bv & 2u) && __uint_as_float(xv.y) == mf) j = 1;
      if ((bv & 1u) && __uint_as_float(xv.x) == mf) j = 0;
    } else {
      const uint32_t h = V::from_f32(mf);
      m2 = h | (h << 16);
      uint32_t m01, m23, m45, m67;
      expand8_16(bv, m01, m23, m45, m67);
      // element j of the vector owns 16-bit lane j of the 64-bit words q (j < 4), r
      const uint32_t q0 = V::eq_mask(xv.x, m2) & m01;
      const uint32_t q1 = V::eq_mask(xv.y, m2) & m23;
      const uint32_t q2 = V::eq_mask(xv.z, m2) & m45;
      const uint32_t q3 = V::eq_mask(xv.w, m2) & m67;
      const unsigned long long q = (unsigned long long)q0 | ((unsigned long long)q1 << 32);
      const unsigned long long r = (unsigned long long)q2 | ((unsigned long long)q3 << 32);
      j = q ? (__ffsll((long long)q) - 1) >> 4 : 4 + ((__ffsll((long long)r) - 1) >> 4);
    }
    j = __shfl_sync(kFull, j, wl);
    return e0 + (uint32_t)((wk * 32 + wl) * E + j);
  }
};

// Masked maximum and its lowest index over elements [e0, e1) of one row, by one warp.
template <int DT, int UNROLL>
__device__ __forceinline__ Partial scan_warp_fast(const void* row_base, const uint32_t* mrow,
                                                  int64_t e0, int64_t e1, int lane) {
  WarpSegment<DT, UNROLL> seg;
  seg.load(row_base, mrow, e0, e1, lane);
  const uint32_t M = seg.max_code();
  Partial part;
  part.flags = M ? kFlagAny : 0u;
  part.ord = M;
  part.idx = (M == 0u || M == kOrd32NaN) ? 0xFFFFFFFFu : seg.first_index(M);
  return part;
}

// ---------------------------------------------------------------------------------------
// generic path: any alignment, and f64. Scalar coalesced loads; phase 2 re-reads the
// segment (it is still in L1/L2).
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

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(kFull, v, o);
    v = other > v ? other : v;
  }
  return v;
}

// One warp's segment [e0, e1) on the generic path: coalesced scalar loads, any alignment,
// any dtype; first_index re-reads the segment (it is still in L1/L2).
template <int DT>
struct GenericSegment {
  const void* row;
  const uint32_t* mrow;
  int64_t e0, e1;
  int lane;
  unsigned long long tbest;  // lane maximum as an order code, 0 = no valid token

  __device__ __forceinline__ void load(const void* row_base, const uint32_t* mrow_, int64_t e0_,
                                       int64_t e1_, int lane_) {
    row = row_base;
    mrow = mrow_;
    e0 = e0_;
    e1 = e1_;
    lane = lane_;
  }

  __device__ __forceinline__ uint32_t bit(int64_t e) const {
    return mrow ? ((__ldg(mrow + (e >> 5)) >> (e & 31)) & 1u) : 1u;
  }

  __device__ __forceinline__ unsigned long long max_code() {
    tbest = 0ull;
    for (int64_t e = e0 + lane; e < e1; e += 32) {
      if (bit(e)) {
        const unsigned long long o = elem_ord<DT>(load_elem<DT>(row, e));
        tbest = o > tbest ? o : tbest;
      }
    }
    return warp_max_u64(tbest);
  }

  __device__ __forceinline__ uint32_t first_index(unsigned long long M) {
    uint32_t cand = 0xFFFFFFFFu;
    if (tbest == M) {
      for (int64_t e = e0 + lane; e < e1; e += 32) {
        if (bit(e) && elem_ord<DT>(load_elem<DT>(row, e)) == M) {
          cand = (uint32_t)e;
          break;
        }
      }
    }
    return __reduce_min_sync(kFull, cand);
  }
};

template <int DT>
__device__ __forceinline__ Partial scan_warp_generic(const void* row_base, const uint32_t* mrow,
                                                     int64_t e0, int64_t e1, int lane) {
  GenericSegment<DT> seg;
  seg.load(row_base, mrow, e0, e1, lane);
  const unsigned long long M = seg.max_code();
  const unsigned long long nan_code = (DT == kF64) ? kOrd64NaN : (unsigned long long)kOrd32NaN;
  Partial part;
  part.flags = M ? kFlagAny : 0u;
  part.ord = M;
  part.idx = (M == 0ull || M == nan_code) ? 0xFFFFFFFFu : seg.first_index(M);
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
  __stcg(reinterpret_cast<ulonglong2*>(p), w);
}

__device__ __forceinline__ Partial warp_merge(Partial acc) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Partial other;
    other.ord = __shfl_xor_sync(kFull, acc.ord, o);
    other.idx = __shfl_xor_sync(kFull, acc.idx, o);
    other.flags = __shfl_xor_sync(kFull, acc.flags, o);
    merge(acc, other);
  }
  return acc;
}

// Combined result of member row `i` of a group: its `segs` partials, merged by one warp.
// The partials are read once and zeroed, so every call leaves the workspace zero-filled
// whatever layout the next call uses.
__device__ __forceinline__ Partial reduce_member(Partial* base, int segs, int lane) {
  Partial acc = empty_partial();
  for (int s = lane; s < segs; s += 32) {
    merge(acc, ld_partial_cg(base + s));
    __stcg(reinterpret_cast<ulonglong2*>(base + s), make_ulonglong2(0ull, 0ull));
  }
  return warp_merge(acc);
}

// Outputs of one group, computed by one warp. `single` is the only partial when a group
// has a single segment (no workspace).
template <int MODE, bool IS64>
__device__ __forceinline__ void finalize_group(const ScanParams& p, int64_t group,
                                               const Partial* single, int lane, int parts) {
  const int P = p.per_group;
  Partial* base = single ? nullptr : p.ws_part + group * (int64_t)P * parts;
  if constexpr (MODE == kModeArgmax || MODE == kModeKey) {
    const Partial r = single ? *single : reduce_member(base, parts, lane);
    if (lane != 0) return;
    if constexpr (MODE == kModeArgmax) {
      decode_partial(r, IS64, &p.out_idx[group], &p.out_status[group]);
    } else {
      unsigned long long key = 0ull;
      if (r.flags & kFlagAny) key = (r.ord << 32) | (unsigned long long)(0xFFFFFFFFu - r.idx);
      if (r.flags & kFlagWaitTimeout) key = kKeyWaitTimeout;
      if (p.n_key_dst) {
        if (__ldcg(p.key_failed) == 0ull) {
          const int64_t slot =
              ((__ldcg(p.key_epoch) + 1ull) & 1ull ? p.key_parity_stride : 0) + group;
          for (int i = 0; i < p.n_key_dst; ++i) p.key_dst[i][slot] = key;
        }
      } else {
        p.out_key[group] = key;
      }
    }
  } else {
    // speculative verify: members in position order; the first row that differs from
    // its draft (or carries a status) decides. Every member is reduced even after the
    // decision, so that all partials are zeroed.
    const int G = P - 1;
    int32_t acc = G, corr = -1;
    uint32_t st = 0u;
    bool decided = false;
    for (int i = 0; i < P; ++i) {
      const Partial r = single ? *single : reduce_member(base + (int64_t)i * parts, parts, lane);
      if (decided) continue;
      int32_t sel;
      uint32_t rs;
      decode_partial(r, IS64, &sel, &rs);
      if (i < G) {
        if (rs) {
          acc = i;
          st = rs;
          decided = true;
        } else if (sel != __ldg(p.drafts + group * p.draft_stride + i)) {
          acc = i;
          corr = sel;
          decided = true;
        }
      } else if (p.bonus) {
        if (rs) {
          st = rs;
        } else {
          corr = sel;
        }
      }
    }
    if (lane == 0) {
      p.accept_len[group] = acc;
      p.correction[group] = corr;
      p.out_status[group] = st;
    }
  }
}

// Speculative-verify outputs of one group whose rows left one partial each (the cluster
// path), for groups of at most 32 rows: lane i reads row i's partial and draft token, so
// all rows are read in one round trip, and ballots find the first row that decides. Same
// decisions as finalize_group's member loop; the partials are zeroed after reading.
template <bool IS64>
__device__ void finalize_verify_rows(const ScanParams& p, uint32_t group, int lane) {
  const int P = p.per_group, G = P - 1;
  Partial* base = p.ws_part + (int64_t)group * P;
  Partial r = empty_partial();
  int32_t draft = 0;
  if (lane < P) {
    r = ld_partial_cg(base + lane);
    __stcg(reinterpret_cast<ulonglong2*>(base + lane), make_ulonglong2(0ull, 0ull));
    if (lane < G) draft = __ldg(p.drafts + (int64_t)group * p.draft_stride + lane);
  }
  int32_t sel = -1;
  uint32_t rs = 0u;
  if (lane < P) decode_partial(r, IS64, &sel, &rs);
  // first draft position whose row carries a status or selects another token
  const unsigned miss = __ballot_sync(kFull, lane < G && (rs != 0u || sel != draft));
  const int acc = miss ? __ffs(miss) - 1 : G;
  const int32_t sel_d = __shfl_sync(kFull, sel, acc);
  const uint32_t rs_d = __shfl_sync(kFull, rs, acc);
  if (lane == 0) {
    int32_t corr = -1;
    uint32_t st = 0u;
    if (acc < G || p.bonus) {  // a mismatch's replacement, or the bonus from row G
      if (rs_d) {
        st = rs_d;
      } else {
        corr = sel_d;
      }
    }
    p.accept_len[group] = acc;
    p.correction[group] = corr;
    p.out_status[group] = st;
  }
}

// Release the warp's partial and take a ticket; true for the warp that completes a group.
__device__ __forceinline__ bool take_ticket(Partial* slot, const Partial& part, uint32_t* counter,
                                            uint32_t total, int lane) {
  uint32_t t = 0u;
  if (lane == 0) {
    st_partial(slot, part);
    // release this warp's partial and draw a ticket in one acq_rel atomic
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(t) : "l"(counter) : "memory");
  }
  t = __shfl_sync(kFull, t, 0);
  const bool last = (t == total - 1u);
  if (last) {
    // every lane of the finishing warp reads partials released by other warps
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (lane == 0) *counter = 0u;  // ready for the next call
  }
  return last;
}

template <int DT, bool FAST, int MODE, int MAXWARPS, int UNROLL>
__global__ void __launch_bounds__(MAXWARPS * 32)
    masked_select_kernel(const ScanParams p) {
  __shared__ Partial s_part[MAXWARPS];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const uint32_t row = blockIdx.x / (uint32_t)p.ctas_per_row;
  const int cta = (int)(blockIdx.x - row * (uint32_t)p.ctas_per_row);
  const int seg = cta * nwarps + warp;
  // rows per group exceed one only when verifying
  const uint32_t group = (MODE == kModeVerify) ? row / (uint32_t)p.per_group : row;
  const uint32_t member = row - group * (uint32_t)p.per_group;

  // Programmatic dependent launch: everything this kernel reads may come from the
  // preceding kernel in the stream.
  asm volatile("griddepcontrol.wait;" ::: "memory");
#if ONYX_PDL_EARLY
  asm volatile("griddepcontrol.launch_dependents;" :::);
#endif

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

  Partial part = empty_partial();
  if (bad_state) {
    part.flags = kFlagBadState;
  } else if (seg < p.segs) {  // warp-uniform
    const int64_t e0 = (int64_t)seg * p.seg_elems;
    const int64_t e1 = min(e0 + p.seg_elems, p.vocab);
    if constexpr (FAST) {
      part = scan_warp_fast<DT, UNROLL>(row_base, mrow, e0, e1, lane);
    } else {
      part = scan_warp_generic<DT>(row_base, mrow, e0, e1, lane);
    }
    if (part.idx != 0xFFFFFFFFu) part.idx += (uint32_t)p.idx_offset;
  }

#if !ONYX_PDL_EARLY
  // let the next kernel in the stream start its prologue
  asm volatile("griddepcontrol.launch_dependents;" :::);
#endif

  // merge the CTA's warp partials in shared memory; warp 0 carries the result on
  if (nwarps > 1) {
    if (lane == 0) s_part[warp] = part;
    __syncthreads();
    if (warp != 0) return;
    part = warp_merge(lane < nwarps ? s_part[lane] : empty_partial());
  }

  const uint32_t total = (uint32_t)(p.per_group * p.ctas_per_row);
  if (total == 1u) {
    finalize_group<MODE, DT == kF64>(p, group, &part, lane, p.ctas_per_row);
    return;
  }
  if (take_ticket(p.ws_part + blockIdx.x, part, p.ws_count + group, total, lane))
    finalize_group<MODE, DT == kF64>(p, group, nullptr, lane, p.ctas_per_row);
}

// Cluster kernel: the CTAs of one thread-block cluster split one row between them (one
// warp per segment):
//   1. every warp loads its segment and computes the segment maximum;
//   2. after a CTA barrier every warp knows the CTA maximum;
//   3. only warps whose own maximum equals it search their registers for its lowest index
//      (normally one warp per CTA), and a second CTA barrier publishes the result;
//   4. each CTA writes its (maximum, lowest index) into rank 0's shared memory through
//      distributed shared memory, followed by the one cluster barrier;
//   5. rank 0 takes the largest maximum and the lowest index among the CTAs holding it
//      and writes the row's outputs.
// No atomics, no fences, no workspace. Used for the argmax / gather / shard-key modes when
// a row needs at most kMaxClusterCtas x kMaxClusterWarps warp segments.
constexpr int kMaxClusterCtas = 8;

// ---- mbarrier helpers (cluster path) ---------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// The waiting warp is parked by the hardware until the phase completes or the hint (ns)
// passes, instead of polling.
__device__ __forceinline__ bool mbar_try_wait_cluster(unsigned long long* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return done != 0u;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __noinline__ bool mbar_wait_cluster_slow(unsigned long long* bar, uint32_t parity,
                                                    unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait_cluster(bar, parity))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}

// Waits for phase `parity` of `bar` to complete; gives up (false) after `limit_ns`. The
// first poll is inline: normally the phase is already complete.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(unsigned long long* bar,
                                                          uint32_t parity,
                                                          unsigned long long limit_ns) {
  return mbar_try_wait_cluster(bar, parity) || mbar_wait_cluster_slow(bar, parity, limit_ns);
}

// Asynchronous 8-byte store into another CTA's shared memory (both addresses from mapa, in
// the same CTA) whose completion is counted on that CTA's mbarrier.
__device__ __forceinline__ void st_async_u64(uint32_t remote_addr, unsigned long long v,
                                             uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.u64 [%0], %1, [%2];" ::"r"(
          remote_addr),
      "l"(v), "r"(remote_bar)
      : "memory");
}

__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}

constexpr unsigned long long kClusterWaitLimitNs = 500ull * 1000ull * 1000ull;  // 0.5 s

// Whether row `row`'s DFA state id (gather mode) lies outside the table.
__device__ __forceinline__ bool row_bad_state(const ScanParams& p, uint32_t row) {
  if (!p.mask || !p.state_ids) return false;
  const int32_t s = __ldg(p.state_ids + row);
  return (s < 0) || ((int64_t)s >= p.n_states);
}

// Where row `row` and its mask live; nullptr logits for a row whose DFA state id is out
// of range. Rows are group-major; groups hold more than one row only when verifying.
template <int DT, int MODE>
__device__ __forceinline__ void locate_row(const ScanParams& p, uint32_t row, const void** base,
                                           const uint32_t** mrow) {
  using St = typename Elem<DT>::storage;
  if constexpr (MODE == kModeVerify) {
    const uint32_t group = row / (uint32_t)p.per_group;
    const uint32_t member = row - group * (uint32_t)p.per_group;
    *base = static_cast<const St*>(p.logits) + (int64_t)group * p.group_stride +
            (int64_t)member * p.row_stride;
    *mrow = p.mask + (int64_t)group * p.mask_group_stride + (int64_t)member * p.mask_row_stride;
    return;
  }
  *base = static_cast<const St*>(p.logits) + (int64_t)row * p.group_stride;
  *mrow = nullptr;
  if (p.mask) {
    if (p.state_ids) {
      const int32_t s = __ldg(p.state_ids + row);
      if ((s < 0) || ((int64_t)s >= p.n_states)) {
        *base = nullptr;
      } else {
        *mrow = p.mask + (int64_t)s * p.mask_row_stride;
      }
    } else {
      *mrow = p.mask + (int64_t)row * p.mask_group_stride;
    }
  }
}

template <int DT, int MODE, int MAXWARPS, class Seg>
__device__ __forceinline__ void cluster_select(const ScanParams& p) {
  static_assert(DT != kF64, "f64 order codes do not pack with an index");
  __shared__ uint32_t s_wmax[MAXWARPS];
  __shared__ uint32_t s_widx[MAXWARPS];
  __shared__ unsigned long long s_key[kMaxClusterCtas];  // rank 0: every CTA's key
  __shared__ unsigned long long s_keys_bar;  // rank 0: completes once every key has landed
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  uint32_t rank, row;  // one cluster per row
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  asm("mov.u32 %0, %%clusterid.x;" : "=r"(row));
  const int C = p.ctas_per_row;  // cluster size
  const int seg_id = (int)rank * nwarps + warp;

  if (rank == 0 && threadIdx.x == 0) {
    mbar_init(&s_keys_bar, 1u);  // rank 0's own arrive, plus the other CTAs' key bytes
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  // First phase of the cluster barrier: its completion guarantees every CTA of the cluster
  // is running and rank 0's mbarrier is initialised, before any access to another CTA's
  // shared memory (step 4). It is awaited while the segment's loads are in flight.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const void* row_base;
  const uint32_t* mrow;
  locate_row<DT, MODE>(p, row, &row_base, &mrow);

  // 1. segment maximum
  Seg seg;
  const bool active = row_base != nullptr && seg_id < p.segs;  // warp-uniform
  uint32_t wmax = 0u;
  if (active) {
    const int64_t e0 = (int64_t)seg_id * p.seg_elems;
    seg.load(row_base, mrow, e0, min(e0 + p.seg_elems, p.vocab), lane);
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  if (active) wmax = (uint32_t)seg.max_code();
  asm volatile("griddepcontrol.launch_dependents;" :::);

  // 2. CTA maximum, known to every warp after one CTA barrier
  if (lane == 0) s_wmax[warp] = wmax;
  __syncthreads();
  const uint32_t cmax = __reduce_max_sync(kFull, lane < nwarps ? s_wmax[lane] : 0u);

  // 3. lowest index of the CTA maximum, searched by the warps that hold it
  uint32_t widx = 0xFFFFFFFFu;
  if (active && wmax == cmax && cmax != 0u && cmax != kOrd32NaN) widx = seg.first_index(cmax);
  if (lane == 0) s_widx[warp] = widx;
  __syncthreads();

  // 4. each CTA's key (maximum << 32 | ~lowest index) into rank 0's shared memory: rank 0
  //    stores its own; every other CTA stores asynchronously, the store's completion counted
  //    on rank 0's mbarrier, which completes once every key has landed
  if (warp == 0) {
    const uint32_t cidx = __reduce_min_sync(kFull, lane < nwarps ? s_widx[lane] : 0xFFFFFFFFu);
    if (lane == 0) {
      const unsigned long long key = ((unsigned long long)cmax << 32) | (0xFFFFFFFFu - cidx);
      if (rank == 0) {
        s_key[0] = key;
        mbar_arrive_expect_tx(&s_keys_bar, (uint32_t)(C - 1) * 8u + p.withheld_key_bytes);
      } else {
        st_async_u64(map_to_rank(&s_key[rank], 0u), key, map_to_rank(&s_keys_bar, 0u));
      }
    }
  }

  // 5. outputs: the largest key among the CTAs is the row maximum at its lowest index
  bool keys_landed = true;
  if (rank == 0 && warp == 0)
    keys_landed = __all_sync(kFull, mbar_wait_cluster_bounded(&s_keys_bar, 0u, kClusterWaitLimitNs));
  // Second phase of the cluster barrier: keeps the other CTAs running until rank 0 holds
  // their keys.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  if (rank == 0 && warp == 0) {
    const unsigned long long key = lane < C ? s_key[lane] : 0ull;
    const uint32_t M = __reduce_max_sync(kFull, (uint32_t)(key >> 32));
    const uint32_t low = __reduce_max_sync(kFull, (uint32_t)(key >> 32) == M ? (uint32_t)key : 0u);
    const uint32_t idx = 0xFFFFFFFFu - low;
    Partial part;
    part.flags = (row_bad_state(p, row) ? kFlagBadState : 0u) | (M ? kFlagAny : 0u) |
                 (keys_landed ? 0u : kFlagWaitTimeout);
    part.ord = M;
    part.idx = idx == 0xFFFFFFFFu ? idx : idx + (uint32_t)p.idx_offset;
    if constexpr (MODE == kModeVerify) {
      // the row's result joins its group through one ticket per row; the last row of the
      // group decides acceptance
      const uint32_t group = row / (uint32_t)p.per_group;
      if (take_ticket(p.ws_part + row, part, p.ws_count + group, (uint32_t)p.per_group, lane)) {
        if (p.per_group <= 32) {
          finalize_verify_rows<false>(p, group, lane);
        } else {
          finalize_group<MODE, false>(p, group, nullptr, lane, 1);
        }
      }
    } else {
      finalize_group<MODE, false>(p, row, &part, lane, 1);
    }
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

template <int DT, bool FAST, int MODE, int MAXWARPS, int UNROLL>
__global__ void __launch_bounds__(MAXWARPS * 32, 1024 / (MAXWARPS * 32))
    masked_select_cluster_kernel(const ScanParams p) {
  if constexpr (FAST) {
    cluster_select<DT, MODE, MAXWARPS, WarpSegment<DT, UNROLL>>(p);
  } else {
    cluster_select<DT, MODE, MAXWARPS, GenericSegment<DT>>(p);
  }
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
    expand8_16(bits, m01, m23, m45, m67);
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
  pr.flags = (best == kKeyWaitTimeout ? kFlagWaitTimeout : 0u) | (best ? kFlagAny : 0u);
  pr.ord = best >> 32;
  pr.idx = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
  decode_partial(pr, false, &out_idx[r], &out_status[r]);
}

#include "peer_exchange.cuh"
#include "dfa_masks.cuh"
#include "masked_sample.cuh"
#include "masked_sample_cluster.cuh"

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
#ifndef ONYX_THREADS
#define ONYX_THREADS 256
#endif
#ifndef ONYX_UNROLL
#define ONYX_UNROLL 8
#endif
constexpr int kThreads = ONYX_THREADS;
constexpr int kUnroll = ONYX_UNROLL;
constexpr int kWarpsPerBlock = kThreads / 32;
constexpr int kGenericPerLane = 32;  // generic path: 1,024 elements per warp segment

static thread_local int g_last_cuda_error = 0;

struct Plan {
  bool fast;
  int64_t seg_elems;
  int segs;          // warp segments per row
  int warps;         // warps per CTA
  int ctas_per_row;  // CTAs per row
};

static int vec_elems(int dt) { return dt == kF32 ? 4 : 8; }

static Plan make_plan(int dt, int64_t vocab, bool aligned) {
  Plan pl;
  pl.fast = aligned && (dt == kF32 || dt == kF16 || dt == kBF16);
  // one segment per warp
  pl.seg_elems = pl.fast ? (int64_t)32 * kUnroll * vec_elems(dt) : (int64_t)32 * kGenericPerLane;
  pl.segs = (int)((vocab + pl.seg_elems - 1) / pl.seg_elems);
  pl.warps = pl.segs < kWarpsPerBlock ? pl.segs : kWarpsPerBlock;
  pl.ctas_per_row = (pl.segs + pl.warps - 1) / pl.warps;
  return pl;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static size_t workspace_bytes_for(int64_t rows, int64_t groups, const Plan& pl, int per_group) {
  if ((int64_t)pl.ctas_per_row * per_group == 1) return 0;
  return align_up((size_t)rows * pl.ctas_per_row * sizeof(Partial), 256) +
         align_up((size_t)groups * sizeof(uint32_t), 256);
}

template <int DT, bool FAST, int MODE>
static cudaError_t launch_t(const ScanParams& p, cudaStream_t stream, bool pdl) {
  const int64_t blocks = p.rows * p.ctas_per_row;
  const int warps = (p.segs + p.ctas_per_row - 1) / p.ctas_per_row;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3((unsigned)(32 * warps), 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, masked_select_kernel<DT, FAST, MODE, kWarpsPerBlock, kUnroll>, p);
}

constexpr int kMaxClusterWarps = 16;

// Cluster layout for one row: at most kMaxClusterCtas CTAs of at most kMaxClusterWarps warps,
// one warp per segment. False when the row needs more (the ticket kernel handles it).
static bool cluster_layout(int segs, int* ctas, int* warps) {
  if (segs < 1 || segs > kMaxClusterCtas * kMaxClusterWarps) return false;
  int w = segs < kWarpsPerBlock ? segs : kWarpsPerBlock;
  int c = (segs + w - 1) / w;
  if (c > kMaxClusterCtas) {
    c = kMaxClusterCtas;
    w = (segs + c - 1) / c;
  }
  *ctas = c;
  *warps = w;
  return true;
}

// ---- process-wide options (onyx_set_option) --------------------------------------------
// Read from the environment once, at the first use of any option; changed afterwards only
// through onyx_set_option. Launches read them without a lock.
struct Options {
  std::atomic<int64_t> v[ONYX_OPTION_COUNT];
};

static int64_t env_int(const char* name, int64_t dflt) {
  const char* s = getenv(name);
  return (s && *s) ? (int64_t)strtoll(s, nullptr, 10) : dflt;
}

static int64_t env_sample_form() {
  const char* s = getenv("ONYX_B200_SAMPLE_FORM");
  if (!s) return 0;
  if (strcmp(s, "single") == 0) return -1;
  if (strncmp(s, "cluster:", 8) == 0) return atoi(s + 8);
  return 0;
}

static Options& options() {
  static Options* o = [] {
    Options* x = new Options;
    for (auto& a : x->v) a.store(0);
    x->v[ONYX_OPTION_CLUSTER].store(env_int("ONYX_B200_CLUSTER", 1) != 0 ? 1 : 0);
    x->v[ONYX_OPTION_PDL].store(env_int("ONYX_B200_PDL", 1) != 0 ? 1 : 0);
    x->v[ONYX_OPTION_SAMPLE_FORM].store(env_sample_form());
    return x;
  }();
  return *o;
}

static int64_t option(int id) { return options().v[id].load(std::memory_order_relaxed); }

// Test hook for the bounded waits of the cluster path: key bytes rank 0 expects beyond
// those sent (0 in normal use).
static uint32_t withheld_key_bytes() {
  return (uint32_t)option(ONYX_OPTION_TEST_WITHHELD_KEY_BYTES) & 0xFFFFu;
}

static bool cluster_enabled() { return option(ONYX_OPTION_CLUSTER) != 0; }

template <int DT, bool FAST, int MODE>
static cudaError_t launch_cluster_t(const ScanParams& p, int warps, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.rows * p.ctas_per_row), 1, 1);
  cfg.blockDim = dim3((unsigned)(32 * warps), 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.ctas_per_row;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(
      &cfg, masked_select_cluster_kernel<DT, FAST, MODE, kMaxClusterWarps, kUnroll>, p);
}

// Launches the cluster kernel when the row fits one cluster; returns false otherwise.
template <int MODE>
static bool dispatch_cluster(int dt, bool fast, ScanParams& p, cudaStream_t s, bool pdl,
                             cudaError_t* err) {
  {
    int ctas = 0, warps = 0;
    if (!cluster_enabled() || (MODE != kModeVerify && p.per_group != 1) ||
        !cluster_layout(p.segs, &ctas, &warps))
      return false;
    // f64 order codes are 64-bit and do not pack with an index: the ticket merge serves it
    if (dt == kF64) return false;
    if (p.rows * (int64_t)ctas > 0x7FFFFFFFll) return false;
    p.ctas_per_row = ctas;
    p.withheld_key_bytes = withheld_key_bytes();
    switch (dt) {
      case kBF16:
        *err = fast ? launch_cluster_t<kBF16, true, MODE>(p, warps, s, pdl)
                    : launch_cluster_t<kBF16, false, MODE>(p, warps, s, pdl);
        return true;
      case kF16:
        *err = fast ? launch_cluster_t<kF16, true, MODE>(p, warps, s, pdl)
                    : launch_cluster_t<kF16, false, MODE>(p, warps, s, pdl);
        return true;
      case kF32:
        *err = fast ? launch_cluster_t<kF32, true, MODE>(p, warps, s, pdl)
                    : launch_cluster_t<kF32, false, MODE>(p, warps, s, pdl);
        return true;
    }
    return false;
  }
}

template <int MODE>
static cudaError_t dispatch(int dt, bool fast, const ScanParams& p, cudaStream_t s, bool pdl) {
  // kernels index rows and CTAs in 32 bits; a grid never exceeds rows x segments blocks
  if (p.rows * (int64_t)p.segs > 0x7FFFFFFFll) return cudaErrorInvalidValue;
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

static bool pdl_enabled() { return option(ONYX_OPTION_PDL) != 0; }

static int bind_workspace(ScanParams& p, void* ws, size_t ws_bytes, size_t need,
                          int64_t groups) {
  if (need == 0) {
    p.ws_part = nullptr;
    p.ws_count = nullptr;
    return ONYX_OK;
  }
  if (!ws || ws_bytes < need || ((uintptr_t)ws & 255u)) return ONYX_ERR_WORKSPACE;
  const size_t part_bytes = align_up((size_t)p.rows * p.ctas_per_row * sizeof(Partial), 256);
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

int onyx_set_option(int id, int64_t value) {
  if (id < 0 || id >= ONYX_OPTION_COUNT) return ONYX_ERR_INVALID_ARGUMENT;
  switch (id) {
    case ONYX_OPTION_CLUSTER:
    case ONYX_OPTION_PDL:
      if (value != 0 && value != 1) return ONYX_ERR_INVALID_ARGUMENT;
      break;
    case ONYX_OPTION_SAMPLE_FORM:
      if (value < -1 || value > kCsMaxCluster) return ONYX_ERR_INVALID_ARGUMENT;
      break;
    case ONYX_OPTION_TEST_WITHHELD_KEY_BYTES:
      if (value < 0 || value > 0xFFFF) return ONYX_ERR_INVALID_ARGUMENT;
      break;
  }
  options().v[id].store(value);
  return ONYX_OK;
}

int64_t onyx_get_option(int id) {
  if (id < 0 || id >= ONYX_OPTION_COUNT) return -1;
  return option(id);
}

int onyx_last_cuda_error(void) { return g_last_cuda_error; }

const char* onyx_error_string(int code) {
  switch (code) {
    case ONYX_OK: return "ok";
    case ONYX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ONYX_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case ONYX_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case ONYX_ERR_CUDA: return "CUDA launch failed (see onyx_last_cuda_error)";
    case ONYX_ERR_SCRATCH_LIMIT:
      return "request needs more than the library's fixed no-alloc scratch "
             "(ONYX_NOALLOC_SCRATCH_BYTES); use onyx_masked_argmax with a workspace";
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
  p.ctas_per_row = pl.ctas_per_row;
  p.seg_elems = pl.seg_elems;
  p.out_idx = out_idx;
  p.out_status = out_status;
  cudaError_t cluster_err = cudaSuccess;
  if (dispatch_cluster<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled(),
                                    &cluster_err))
    return finish_launch(cluster_err);  // one cluster per row: no workspace involved
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
  p.ctas_per_row = pl.ctas_per_row;
  p.seg_elems = pl.seg_elems;
  p.out_idx = out_idx;
  p.out_status = out_status;
  cudaError_t cluster_err = cudaSuccess;
  if (dispatch_cluster<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled(),
                                    &cluster_err))
    return finish_launch(cluster_err);  // one cluster per row: no workspace involved
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
  p.ctas_per_row = pl.ctas_per_row;
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
  // one cluster per row, rows joined per group by a ticket; uses the first `rows`
  // partials of the workspace bound above for the ticket layout
  cudaError_t cluster_err = cudaSuccess;
  if (dispatch_cluster<kModeVerify>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled(),
                                    &cluster_err))
    return finish_launch(cluster_err);
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
  p.ctas_per_row = pl.ctas_per_row;
  p.seg_elems = pl.seg_elems;
  p.out_key = reinterpret_cast<unsigned long long*>(out_keys);
  cudaError_t cluster_err = cudaSuccess;
  if (dispatch_cluster<kModeKey>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled(),
                                    &cluster_err))
    return finish_launch(cluster_err);  // one cluster per row: no workspace involved
  rc = bind_workspace(p, workspace, workspace_bytes, workspace_bytes_for(rows, rows, pl, 1), rows);
  if (rc) return rc;
  return finish_launch(dispatch<kModeKey>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}

// ---- masked sampling: cluster form ------------------------------------------------------

// ONYX_OPTION_SAMPLE_FORM (a diagnostic and test switch): -1 runs the one-CTA-per-row
// kernel for every shape; k >= 1 asks for k CTAs per row (raised to the least k whose
// shared memory holds a row); 0 (default): the cluster form with k chosen from the batch
// size, wherever a row fits.
static int sample_form() {
  const int64_t v = option(ONYX_OPTION_SAMPLE_FORM);
  if (v == -1) return -1;
  if (v >= 1 && v <= kCsMaxCluster) return (int)v;
  return 0;
}

constexpr int kNoClusterPlan = -1000;

struct ClusterSamplePlan {
  int k = 0, slice = 0, off_words = 0, off_work = 0, off_comb = 0;
  size_t smem = 0;
};

static size_t cs_align16(size_t x) { return (x + 15) & ~(size_t)15; }

// shared memory of the cluster form with k CTAs per row (0: it cannot fit)
static ClusterSamplePlan cs_layout(int k, int64_t vocab, int dtype, bool masked) {
  const int elem = dtype == kF32 ? 4 : 2;
  ClusterSamplePlan pl;
  const int64_t per = (vocab + k - 1) / k;
  const int64_t slice = (per + kCsSliceAlign - 1) / kCsSliceAlign * kCsSliceAlign;
  if (slice > (1 << 26)) return pl;
  pl.k = k;
  pl.slice = (int)slice;
  size_t off = cs_align16((size_t)slice * elem);
  pl.off_words = (int)off;
  if (masked) off += cs_align16((size_t)slice / 32 * 4);
  pl.off_work = (int)off;
  off += dtype == kBF16 ? (size_t)kVtWorkBytes : sizeof(WarpBuf) * kCsWarps;
  pl.off_comb = (int)off;
  const size_t cap = (size_t)cs_comb_share(dtype, k);
  off += cs_align16(cap * 8) + cs_align16(cap * 4);
  pl.smem = off;
  return pl;
}
static_assert(sizeof(WarpBuf) * kCsWarps >= sizeof(CsHist), "histogram overlays the buffers");

static const void* cs_kernel(int dtype) {
  return dtype == kBF16 ? (const void*)masked_sample_cluster_kernel<kBF16>
         : dtype == kF16 ? (const void*)masked_sample_cluster_kernel<kF16>
                         : (const void*)masked_sample_cluster_kernel<kF32>;
}

// Launches the cluster form, or returns kNoClusterPlan when no cluster of at most 16 CTAs
// holds a row in shared memory (the caller then runs the one-CTA kernel).
static int launch_cluster_sample(int dtype, const SampleParams& sp, int dev, cudaStream_t stream,
                                 int forced_k) {
  struct DevInfo {
    bool ready = false;
    int sms = 0, max_dyn = 0;
    int fits[3][kCsMaxCluster + 1];  // per dtype and k: resident clusters, -1 not yet asked
  };
  static std::mutex mu;
  static DevInfo info[64];
  const int di = dtype == kBF16 ? 0 : dtype == kF16 ? 1 : 2;
  const void* fn = cs_kernel(dtype);
  std::lock_guard<std::mutex> lock(mu);
  DevInfo& d = info[dev];
  if (!d.ready) {
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return finish_launch(e);
    cudaFuncAttributes fa = {};
    e = cudaFuncGetAttributes(&fa, cs_kernel(kBF16));
    if (e != cudaSuccess) return finish_launch(e);
    d.max_dyn = optin - (int)fa.sharedSizeBytes - 1024;  // margin for the other instantiations
    for (const void* f : {cs_kernel(kBF16), cs_kernel(kF16), cs_kernel(kF32)}) {
      e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_dyn);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return finish_launch(e);
    }
    for (auto& r : d.fits)
      for (int& x : r) x = -1;
    d.ready = true;
  }
  const bool masked = sp.mask != nullptr;
  int k_fit = 0;
  for (int k = 1; k <= kCsMaxCluster; ++k) {
    const ClusterSamplePlan pl = cs_layout(k, sp.vocab, dtype, masked);
    if (pl.k && pl.smem <= (size_t)d.max_dyn) {
      k_fit = k;
      break;
    }
  }
  if (!k_fit) return kNoClusterPlan;
  // spread small batches over the SMs, at least 4096 ids per CTA
  int64_t k_par = d.sms / std::max<int64_t>(1, sp.rows);
  k_par = std::min<int64_t>(k_par, (sp.vocab + 4095) / 4096);
  if (forced_k) k_par = forced_k;
  const int k0 = (int)std::max<int64_t>(k_fit, std::min<int64_t>(k_par, kCsMaxCluster));
  if ((int64_t)k0 * sp.rows > 0x7FFFFFFFll) return kNoClusterPlan;
  // clusters that can be resident at once for k CTAs per row (cached per dtype and k)
  auto active = [&](int k) {
    int& n = d.fits[di][k];
    if (n < 0) {
      cudaLaunchConfig_t q = {};
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = (unsigned)k;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.gridDim = dim3((unsigned)k, 1, 1);
      q.blockDim = dim3(kCsThreads, 1, 1);
      q.dynamicSmemBytes = (size_t)d.max_dyn;  // the largest layout: a bound for every shape
      q.attrs = qa;
      q.numAttrs = 1;
      int clusters = 0;
      const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, fn, &q);
      if (e != cudaSuccess) (void)cudaGetLastError();
      n = e == cudaSuccess ? clusters : 0;
    }
    return n;
  };
  // candidates: k0, then the powers of two below it (down to k_fit); the first that holds
  // every row's cluster at once, else the smallest that runs at all
  int cand[8], nc = 0;
  cand[nc++] = k0;
  if (!forced_k)
    for (int kk = 8; kk >= 1; kk >>= 1)
      if (kk < k0 && kk >= k_fit) cand[nc++] = kk;
  int k = 0;
  for (int i = 0; i < nc && !k; ++i)
    if (active(cand[i]) >= sp.rows) k = cand[i];
  for (int i = nc - 1; i >= 0 && !k; --i)
    if (active(cand[i]) >= 1) k = cand[i];
  if (!k) return kNoClusterPlan;
  {
    const ClusterSamplePlan pl = cs_layout(k, sp.vocab, dtype, masked);
    ClusterSampleParams cp = {};
    cp.logits = sp.logits;
    cp.row_stride = sp.row_stride;
    cp.vocab = sp.vocab;
    cp.mask = sp.mask;
    cp.mask_stride = sp.mask_stride;
    cp.temperature = sp.temperature;
    cp.top_p = sp.top_p;
    cp.seed = sp.seed;
    cp.call = sp.call;
    cp.out_idx = sp.out_idx;
    cp.out_status = sp.out_status;
    cp.k = k;
    cp.slice = pl.slice;
    cp.off_words = pl.off_words;
    cp.off_work = pl.off_work;
    cp.off_comb = pl.off_comb;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)k;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(k * sp.rows), 1, 1);
    cfg.blockDim = dim3(kCsThreads, 1, 1);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e;
    switch (dtype) {
      case kBF16: e = cudaLaunchKernelEx(&cfg, masked_sample_cluster_kernel<kBF16>, cp); break;
      case kF16: e = cudaLaunchKernelEx(&cfg, masked_sample_cluster_kernel<kF16>, cp); break;
      default: e = cudaLaunchKernelEx(&cfg, masked_sample_cluster_kernel<kF32>, cp); break;
    }
    return finish_launch(e);
  }
}

int onyx_masked_sample(const void* logits, int dtype, int64_t rows, int64_t vocab,
                       int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                       double temperature, double top_p, uint64_t seed, uint64_t call,
                       int32_t* out_idx, uint32_t* out_status, void* stream) {
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16) return ONYX_ERR_UNSUPPORTED_DTYPE;
  if (rows < 0 || rows > 0x7FFFFFFFll || vocab <= 0 || vocab > 0x7FFFFFFFll - 1)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (!(temperature > 0.0) || !(temperature < INFINITY) || !(top_p > 0.0) || !(top_p <= 1.0))
    return ONYX_ERR_INVALID_ARGUMENT;
  if (rows == 0) return ONYX_OK;
  if (!logits || !out_idx || !out_status || (row_stride < vocab && rows > 1))
    return ONYX_ERR_INVALID_ARGUMENT;
  if (mask && mask_stride < (vocab + 31) / 32 && rows > 1) return ONYX_ERR_INVALID_ARGUMENT;
  SampleParams sp = {};
  sp.logits = logits;
  sp.row_stride = row_stride;
  sp.vocab = vocab;
  sp.mask = mask;
  sp.mask_stride = mask_stride;
  sp.temperature = temperature;
  sp.top_p = top_p;
  sp.seed = seed;
  sp.call = call;
  sp.rows = rows;
  sp.out_idx = out_idx;
  sp.out_status = out_status;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return finish_launch(e);
  if (dev < 0 || dev >= 64) return ONYX_ERR_INVALID_ARGUMENT;
  const int form = sample_form();
  if (form >= 0) {
    const int rc = launch_cluster_sample(dtype, sp, dev, (cudaStream_t)stream, form);
    if (rc != kNoClusterPlan) return rc;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows, 1, 1);
  cfg.blockDim = dim3(kSampleThreads, 1, 1);
  cfg.stream = (cudaStream_t)stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cfg.dynamicSmemBytes = kSampleSmemBytes;
  // the compaction buffers take 48 KB of dynamic shared memory: opt in once per device
  {
    static std::mutex mu;
    static bool ready[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev]) {
      for (const void* fn : {(const void*)masked_sample_kernel<kBF16>,
                             (const void*)masked_sample_kernel<kF16>,
                             (const void*)masked_sample_kernel<kF32>}) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSampleSmemBytes);
        if (e != cudaSuccess) return finish_launch(e);
      }
      ready[dev] = true;
    }
  }
  switch (dtype) {
    case kBF16: e = cudaLaunchKernelEx(&cfg, masked_sample_kernel<kBF16>, sp); break;
    case kF16: e = cudaLaunchKernelEx(&cfg, masked_sample_kernel<kF16>, sp); break;
    default: e = cudaLaunchKernelEx(&cfg, masked_sample_kernel<kF32>, sp); break;
  }
  return finish_launch(e);
}

int onyx_dfa_state_masks(const int32_t* trans, int32_t n_states, int32_t dead,
                         int dead_absorbing, const int32_t* states, int64_t rows,
                         const uint8_t* tok_bytes, int64_t n_bytes, const int64_t* tok_offsets,
                         int64_t vocab, uint32_t* out, int64_t out_stride, void* stream) {
  // n_states * 256 table entries are addressed with 32-bit offsets
  if (!trans || n_states < 1 || n_states > (1 << 23) || dead < 0 || dead >= n_states ||
      rows < 0 || vocab < 1 || vocab > 0x7FFFFFFFll - 1 || !tok_offsets || n_bytes < 0 ||
      (n_bytes > 0 && !tok_bytes) || out_stride < (vocab + 31) / 32)
    return ONYX_ERR_INVALID_ARGUMENT;
  if (rows == 0) return ONYX_OK;
  if (!states || !out) return ONYX_ERR_INVALID_ARGUMENT;
  const int64_t words = (vocab + 31) / 32;
  // the most rows per warp (token bytes loaded once for more walks) that still leaves a few
  // waves of warps
  constexpr int64_t kTargetWarps = 28 * 1024;
  int rpw = kDfaLockstep;
  while (rpw < kDfaMaxRowsPerWarp && words * ((rows + 2 * rpw - 1) / (2 * rpw)) >= kTargetWarps)
    rpw *= 2;
  const int64_t kMaxRowsPerLaunch = (int64_t)65535 * rpw;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  for (int64_t r0 = 0; r0 < rows; r0 += kMaxRowsPerLaunch) {
    const int64_t n = std::min(rows - r0, kMaxRowsPerLaunch);
    DfaParams d = {};
    d.trans = trans;
    d.n_states = n_states;
    d.dead = dead;
    d.dead_absorbing = dead_absorbing ? 1 : 0;
    d.states = states + r0;
    d.rows = n;
    d.tok_bytes = tok_bytes;
    d.n_bytes = n_bytes;
    d.tok_offsets = tok_offsets;
    d.vocab = vocab;
    d.out = out + r0 * out_stride;
    d.out_stride = out_stride;
    d.rows_per_warp = rpw;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((words + kDfaWarpsPerBlock - 1) / kDfaWarpsPerBlock),
                       (unsigned)((n + rpw - 1) / rpw), 1);
    cfg.blockDim = dim3(kDfaWarpsPerBlock * 32, 1, 1);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const int rc = finish_launch(cudaLaunchKernelEx(&cfg, dfa_mask_kernel, d));
    if (rc) return rc;
  }
  return ONYX_OK;
}

size_t onyx_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

size_t onyx_exchange_buffer_bytes(int world, int64_t rows_cap) {
  if (world < 1 || world > kMaxExchangeRanks || rows_cap < 1) return 0;
  return kExchangeFlagBytes + (size_t)2 * world * rows_cap * sizeof(unsigned long long);
}

int onyx_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out) {
  if (!bytes || !dev_ptr || !handle_out) return ONYX_ERR_INVALID_ARGUMENT;
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), ptr);
  if (e != cudaSuccess) {
    if (ptr) cudaFree(ptr);
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  *dev_ptr = ptr;
  return ONYX_OK;
}

int onyx_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return ONYX_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  return ONYX_OK;
}

int onyx_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return ONYX_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  return ONYX_OK;
}

int onyx_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return ONYX_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return ONYX_ERR_CUDA;
  }
  return ONYX_OK;
}

int onyx_vocab_exchange_argmax(const void* logits, int dtype, int64_t rows, int64_t shard_vocab,
                               int64_t row_stride, const uint32_t* mask, int64_t mask_stride,
                               int64_t col_offset, int world, int rank,
                               void* const* exchange_bases, int64_t rows_cap,
                               int32_t* out_idx, uint32_t* out_status, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (dtype == kF64) return ONYX_ERR_UNSUPPORTED_DTYPE;
  int rc = common_checks(logits, dtype, rows, shard_vocab, row_stride);
  if (rc) return rc;
  if (world < 1 || world > kMaxExchangeRanks || rank < 0 || rank >= world || !exchange_bases ||
      rows > rows_cap || !out_idx || !out_status)
    return ONYX_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < world; ++i)
    if (!exchange_bases[i] || ((uintptr_t)exchange_bases[i] & 255u)) return ONYX_ERR_INVALID_ARGUMENT;
  if (rows == 0) return ONYX_OK;
  if (!mask || col_offset < 0 || (col_offset & 31) || col_offset + shard_vocab > 0x7FFFFFFFll - 1)
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
  p.ctas_per_row = pl.ctas_per_row;
  p.seg_elems = pl.seg_elems;
  char* own = static_cast<char*>(exchange_bases[rank]);
  unsigned long long* own_epoch = reinterpret_cast<unsigned long long*>(own + kExchangeEpochOffset);
  p.n_key_dst = world;
  p.key_parity_stride = (int64_t)world * rows_cap;
  p.key_epoch = own_epoch;
  p.key_failed = reinterpret_cast<unsigned long long*>(own + kExchangeFailedOffset);
  ExchangeParams x = {};
  for (int i = 0; i < world; ++i) {
    char* base = static_cast<char*>(exchange_bases[i]);
    p.key_dst[i] = reinterpret_cast<unsigned long long*>(base + kExchangeFlagBytes) +
                   (int64_t)rank * rows_cap;
    x.flag_dst[i] = reinterpret_cast<unsigned long long*>(base) + rank;
  }
  x.own_flags = reinterpret_cast<unsigned long long*>(own);
  x.own_epoch = own_epoch;
  x.own_failed = reinterpret_cast<unsigned long long*>(own + kExchangeFailedOffset);
  x.slots = reinterpret_cast<const unsigned long long*>(own + kExchangeFlagBytes);
  x.parity_stride = (int64_t)world * rows_cap;
  x.world = world;
  x.rows = rows;
  x.rows_cap = rows_cap;
  x.out_idx = out_idx;
  x.out_status = out_status;
  const bool pdl = pdl_enabled();
  cudaError_t err = cudaSuccess;
  if (!dispatch_cluster<kModeKey>(dtype, pl.fast, p, (cudaStream_t)stream, pdl, &err)) {
    rc = bind_workspace(p, workspace, workspace_bytes, workspace_bytes_for(rows, rows, pl, 1), rows);
    if (rc) return rc;
    err = dispatch<kModeKey>(dtype, pl.fast, p, (cudaStream_t)stream, pdl);
  }
  if (err != cudaSuccess) return finish_launch(err);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(1024, 1, 1);
  cfg.stream = (cudaStream_t)stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return finish_launch(cudaLaunchKernelEx(&cfg, exchange_combine_kernel, x));
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

// ---------------------------------------------------------------------------------------
// Allocation-free variant of onyx_masked_argmax.
//
// Who needs it: callers that cannot allocate device memory at the point of the call and
// so cannot hand over a workspace -- e.g. a serving process whose device memory was
// reserved up front by its own pool, a host-language binding that only ever receives
// pointers to buffers someone else allocated, or code running where an allocation would
// synchronise or fail. This entry point takes only inputs and outputs. Rows that fit one
// thread-block cluster need no scratch at all (their CTAs combine in distributed shared
// memory); longer rows, or every row when the cluster option is off, keep their split-row
// partials and tickets in a fixed scratch array compiled into the library.
//
// The array is a file-scope __device__ symbol, so every GPU that loads this library holds
// kNoAllocScratchBytes of it until the process exits. Host code cannot use the symbol's
// name as a device address: the address is looked up with cudaGetSymbolAddress in each
// CUDA context, by the first call that needs the scratch in that context (for the usual
// primary context, the first such call on each device), and kept per context. That first
// call should therefore happen before any stream capture. Every call in a context shares
// the one array: calls whose kernels may overlap on the GPU (different streams, or
// different host threads) race and must be serialised by the caller.
// ---------------------------------------------------------------------------------------
namespace onyx {

constexpr size_t kNoAllocScratchBytes = ONYX_NOALLOC_SCRATCH_BYTES;  // 1 MiB per device
constexpr int kNoAllocMaxContexts = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The calling thread's current driver context, nullptr if there is none (the driver entry
// point is looked up at run time, so the library does not link the driver library).
static CUcontext current_context() {
  static const CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

struct NoAllocEntry {
  CUcontext ctx;
  void* ptr;
};
static std::mutex g_noalloc_mutex;
static NoAllocEntry g_noalloc_cache[kNoAllocMaxContexts] = {};
static int g_noalloc_next = 0;

// Device address of the scratch array in the current context (looked up on first use).
static int noalloc_scratch_address(void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  CUcontext ctx = current_context();
  if (ctx) {
    for (const NoAllocEntry& en : g_noalloc_cache)
      if (en.ctx == ctx && en.ptr) {
        *out = en.ptr;
        return ONYX_OK;
      }
  }
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);  // makes a context current
  if (e != cudaSuccess || ptr == nullptr) {
    g_last_cuda_error = (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    return ONYX_ERR_CUDA;
  }
  if (!ctx) ctx = current_context();
  if (ctx) {
    g_noalloc_cache[g_noalloc_next] = NoAllocEntry{ctx, ptr};
    g_noalloc_next = (g_noalloc_next + 1) % kNoAllocMaxContexts;
  }
  *out = ptr;
  return ONYX_OK;
}

}  // namespace onyx

extern "C" int onyx_masked_argmax_noalloc(const void* logits, int dtype, int64_t rows,
                                          int64_t vocab, int64_t row_stride,
                                          const uint32_t* mask, int64_t mask_stride,
                                          int32_t* out_idx, uint32_t* out_status,
                                          void* stream) {
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
  p.vocab = vocab;
  p.mask = mask;
  p.mask_group_stride = mask_stride;
  p.rows = rows;
  p.per_group = 1;
  p.segs = pl.segs;
  p.ctas_per_row = pl.ctas_per_row;
  p.seg_elems = pl.seg_elems;
  p.out_idx = out_idx;
  p.out_status = out_status;
  // rows that fit one cluster: no scratch
  cudaError_t cluster_err = cudaSuccess;
  if (dispatch_cluster<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled(),
                                    &cluster_err))
    return finish_launch(cluster_err);
  // scratch layout: ticket counters [rows] first, then partials [rows * ctas_per_row]
  const size_t count_bytes = align_up((size_t)rows * sizeof(uint32_t), 256);
  const size_t part_bytes = (size_t)rows * pl.ctas_per_row * sizeof(Partial);
  const bool split = pl.ctas_per_row > 1;
  if (split && count_bytes + part_bytes > kNoAllocScratchBytes) return ONYX_ERR_SCRATCH_LIMIT;
  if (split) {
    void* base = nullptr;
    rc = noalloc_scratch_address(&base);
    if (rc) return rc;
    p.ws_count = static_cast<uint32_t*>(base);
    p.ws_part = reinterpret_cast<Partial*>(static_cast<char*>(base) + count_bytes);
    // the tickets must start at zero whatever an earlier call left behind
    const cudaError_t e =
        cudaMemsetAsync(p.ws_count, 0, (size_t)rows * sizeof(uint32_t), (cudaStream_t)stream);
    if (e != cudaSuccess) {
      g_last_cuda_error = (int)e;
      return ONYX_ERR_CUDA;
    }
  }
  return finish_launch(
      dispatch<kModeArgmax>(dtype, pl.fast, p, (cudaStream_t)stream, pdl_enabled()));
}
