// Shared device helpers for the grammar-masked selection kernels (sm_100a).
//
// Selection contract (bayareahomelander/Onyx, onyx_cuda package):
//   * masked row = allowed values kept, everything else -inf
//     (onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:145-186);
//   * greedy select = first (lowest-index) maximum under float comparison, NaN anywhere in
//     the masked row rejected (onyx_cuda/src/onyx_cuda/torch_backend.py:970-1007);
//   * an all -inf support is rejected (torch_grammar_mask.py:182-185) and an empty support
//     is a grammar no-decision (grammar_selection.py:122-127).
//
// Values are compared through a monotone unsigned "order" code: NaN maps to the maximum
// code (so any NaN in the support surfaces as the row maximum and is reported), -0.0 is
// folded onto +0.0 (so signed zeros tie and the lowest index wins), -inf maps to a small
// non-zero code, and code 0 is reserved for "no support".
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace onyx {

// dtype codes of the C-ABI
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2, kF64 = 3 };

// per-row status bits of the C-ABI
constexpr uint32_t kStatusEmptyMask = 1u;
constexpr uint32_t kStatusAllNegInf = 2u;
constexpr uint32_t kStatusNanInSupport = 4u;
constexpr uint32_t kStatusBadState = 8u;
constexpr uint32_t kStatusWaitTimeout = 16u;

// partial-result flags
constexpr uint32_t kFlagAny = 1u;        // the segment holds at least one valid token
constexpr uint32_t kFlagBadState = 2u;   // the DFA state id of the row is out of range
constexpr uint32_t kFlagAboveNegInf = 4u;  // some valid value is not -inf (mask apply)
constexpr uint32_t kFlagWaitTimeout = 8u;  // a bounded wait for the row's partials gave up
// shard key of a row whose bounded wait gave up: above every real key (a NaN maximum has
// low word 0), so it wins every combine
constexpr unsigned long long kKeyWaitTimeout = ~0ull;

constexpr uint32_t kOrd32NaN = 0xFFFFFFFFu;
constexpr uint32_t kOrd32NegInf = 0x007FFFFFu;  // ord32(-inf)
constexpr unsigned long long kOrd64NaN = 0xFFFFFFFFFFFFFFFFull;
constexpr unsigned long long kOrd64NegInf = 0x000FFFFFFFFFFFFFull;  // ord64(-inf)

__host__ __device__ __forceinline__ uint32_t ord_from_f32_bits(uint32_t u) {
  // caller guarantees u is not a NaN pattern
  if ((u & 0x7FFFFFFFu) == 0u) u = 0u;  // -0.0 -> +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint32_t ord32(float v) {
  if (v != v) return kOrd32NaN;
  return ord_from_f32_bits(__float_as_uint(v));
}

__device__ __forceinline__ unsigned long long ord64(double v) {
  if (v != v) return kOrd64NaN;
  unsigned long long u = (unsigned long long)__double_as_longlong(v);
  if ((u & 0x7FFFFFFFFFFFFFFFull) == 0ull) u = 0ull;
  return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

// A segment's partial result: best order code, its lowest index, flags. 16 bytes.
struct __align__(16) Partial {
  unsigned long long ord;
  uint32_t idx;
  uint32_t flags;
};

__device__ __forceinline__ bool better(unsigned long long ord_a, uint32_t idx_a,
                                       unsigned long long ord_b, uint32_t idx_b) {
  return ord_a > ord_b || (ord_a == ord_b && idx_a < idx_b);
}

// Decode a row's combined partial into (index, status).
__device__ __forceinline__ void decode_partial(const Partial& p, bool is64, int32_t* idx,
                                               uint32_t* status) {
  if (p.flags & kFlagWaitTimeout) {
    *idx = -1;
    *status = kStatusWaitTimeout;
    return;
  }
  if (p.flags & kFlagBadState) {
    *idx = -1;
    *status = kStatusBadState;
    return;
  }
  if (!(p.flags & kFlagAny)) {
    *idx = -1;
    *status = kStatusEmptyMask;
    return;
  }
  const unsigned long long nan_code = is64 ? kOrd64NaN : (unsigned long long)kOrd32NaN;
  const unsigned long long ninf_code = is64 ? kOrd64NegInf : (unsigned long long)kOrd32NegInf;
  if (p.ord == nan_code) {
    *idx = -1;
    *status = kStatusNanInSupport;
    return;
  }
  *idx = (int32_t)p.idx;
  *status = (p.ord == ninf_code) ? kStatusAllNegInf : 0u;
}

// ---------------------------------------------------------------------------------------
// streaming loads: logits are read exactly once, so keep them out of L1 and mark them
// evict-first in L2; mask words are small and re-read by 4-8 neighbouring lanes.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ld_mask_word(const uint32_t* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::evict_last.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// NaN-propagating packed maxima (PTX max.NaN, sm_80+)
__device__ __forceinline__ uint32_t max_nan_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t max_nan_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float max_nan_f32(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// PTX prmt in its default mode: bit 3 of a selector nibble replicates the selected
// byte's most significant bit over the whole byte. (__byte_perm only honours the low
// three bits of each nibble, so it cannot express this.)
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(a), "r"(sel));
  return d;
}

// Expand the 8 mask bits b0..b7 in the low byte of `bits` (higher bits ignored) into
// per-16-bit-lane masks for four packed registers: m01 = [b0 b0 b1 b1] bytes, m23 =
// [b2 b2 b3 b3], m45 = [b4 b4 b5 b5], m67 = [b6 b6 b7 b7] (0x00 or 0xFF each). Bit i
// (i = 0..3) times 0x10204080 has terms at bits i+7, i+14, i+21, i+28, and bit 4+i times
// 0x01020408 at 7+i, 14+i, 21+i, 28+i: in each product the sixteen positions are distinct,
// so nothing carries, and bits 7, 15, 23, 31 hold b0..b3 (b4..b7: the high nibble needs no
// shift first). prmt then sign-replicates the selected bytes.
__device__ __forceinline__ void expand8_16(uint32_t bits, uint32_t& m01, uint32_t& m23,
                                           uint32_t& m45, uint32_t& m67) {
  const uint32_t lo = (bits & 0x0Fu) * 0x10204080u;
  const uint32_t hi = (bits & 0xF0u) * 0x01020408u;
  m01 = prmt_sign(lo, 0x9988u);
  m23 = prmt_sign(lo, 0xBBAAu);
  m45 = prmt_sign(hi, 0x9988u);
  m67 = prmt_sign(hi, 0xBBAAu);
}

// 16-bit float helpers (bit pattern -> float)
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

template <int DT>
struct Elem;
template <>
struct Elem<kF32> {
  using storage = float;
  static constexpr int kBytes = 4;
  __device__ static float to_f32(const storage* p, int64_t i) { return p[i]; }
};
template <>
struct Elem<kF16> {
  using storage = uint16_t;
  static constexpr int kBytes = 2;
  __device__ static float to_f32(const storage* p, int64_t i) { return f16_bits_to_f32(p[i]); }
};
template <>
struct Elem<kBF16> {
  using storage = uint16_t;
  static constexpr int kBytes = 2;
  __device__ static float to_f32(const storage* p, int64_t i) { return bf16_bits_to_f32(p[i]); }
};
template <>
struct Elem<kF64> {
  using storage = double;
  static constexpr int kBytes = 8;
};

inline int dtype_bytes(int dt) {
  switch (dt) {
    case kF32: return 4;
    case kF16: return 2;
    case kBF16: return 2;
    case kF64: return 8;
  }
  return 0;
}

}  // namespace onyx
