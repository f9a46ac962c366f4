// Masked temperature / top-p sampling (included by masked_select.cu inside namespace onyx).
//
// Distribution and top-p set of the reference's sampler, onyx_cuda/src/onyx_cuda/
// selection.py (_filtered_reference_weights): over the valid ids of a row (the grammar mask
// first, as mask.apply leaves invalid ids at -inf), NaN is rejected; if any valid value is
// +inf the +inf ids share the mass equally; otherwise id i weighs exp((v_i - max) / T) in
// float64 (max over the finite valid values), zero weights drop out, probabilities are
// weight / total; ranked by (-probability, id), the shortest prefix whose cumulative
// probability reaches top_p is kept. The draw u in [0, 1) is Philox4x32-10 (key = seed,
// counter = (call, row)) turned into 53 bits; the sampled id is the first kept id, in
// increasing id order, whose cumulative kept probability exceeds u times the kept total.
//
// One CTA of 1024 threads per row. Probability order is value order (exp is monotone and
// one total divides every weight), so the top-p cut is found by a three-level radix select
// on the 32-bit order code of the value (11 + 11 + 10 bits): each level histograms the
// probability mass of the tokens that share the prefix found so far and finds, by a block
// scan from the top, the bin where the mass above reaches top_p. That leaves one exact
// value v*: every token above it is kept, and of the tokens equal to it (in id order) as
// many as the cumulative sum, added one by one as the reference does, needs. Sums over
// many tokens are block reductions, so their rounding differs from the reference's
// sequential sums by a few units in the last place; only a draw or a cumulative within that
// distance of a boundary can come out differently.

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;  // 32: the block scans use one lane per warp
constexpr int kSampleBins = 2048;  // the widest radix level (11 bits)

struct SampleParams {
  const void* logits;
  int64_t row_stride;  // elements
  int64_t vocab;
  const uint32_t* mask;  // nullptr: every id valid
  int64_t mask_stride;   // words
  double temperature;
  double top_p;
  unsigned long long seed;
  unsigned long long call;
  int64_t rows;
  int32_t* out_idx;
  uint32_t* out_status;
};

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC 2011) and the 53-bit double it gives.
__device__ __forceinline__ double philox_uniform(unsigned long long seed, unsigned long long call,
                                                 uint32_t row) {
  uint32_t c0 = (uint32_t)call, c1 = (uint32_t)(call >> 32), c2 = row, c3 = 0u;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
  }
  return ((double)(c0 >> 5) * 67108864.0 + (double)(c1 >> 6)) / 9007199254740992.0;
}

template <int DT>
__device__ __forceinline__ float sample_value(const void* row, int64_t i) {
  if constexpr (DT == kF32) {
    return __ldg(static_cast<const float*>(row) + i);
  } else if constexpr (DT == kBF16) {
    return bf16_bits_to_f32(__ldg(static_cast<const unsigned short*>(row) + i));
  } else {
    return f16_bits_to_f32(__ldg(static_cast<const unsigned short*>(row) + i));
  }
}

__device__ __forceinline__ bool sample_valid(const uint32_t* mrow, int64_t i) {
  return !mrow || ((__ldg(mrow + (i >> 5)) >> (i & 31)) & 1u);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Block-wide sum; every thread gets it. s_red: kSampleWarps doubles.
__device__ __forceinline__ double block_sum_d(double v, double* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  double r = lane < kSampleWarps ? s_red[lane] : 0.0;
  r = warp_sum_d(r);
  __syncthreads();
  return r;
}

// Block-wide exclusive prefix sum in thread order; *total gets the sum.
__device__ __forceinline__ double block_exclusive_scan_d(double v, double* s_red,
                                                         double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  double excl = __shfl_up_sync(kFull, incl, 1);
  if (lane == 0) excl = 0.0;
  if (lane == 31) s_red[warp] = incl;
  __syncthreads();
  double wincl = s_red[lane];  // kSampleWarps == 32: one warp total per lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(kFull, wincl, o);
    if (lane >= o) wincl += n;
  }
  double wexcl = __shfl_up_sync(kFull, wincl, 1);
  if (lane == 0) wexcl = 0.0;
  const double warp_before = __shfl_sync(kFull, wexcl, warp);
  *total = __shfl_sync(kFull, wincl, 31);
  __syncthreads();
  return warp_before + excl;
}

__device__ __forceinline__ uint32_t block_or_u32(uint32_t v, uint32_t* s_u) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_or_sync(kFull, v);
  if (lane == 0) s_u[warp] = v;
  __syncthreads();
  uint32_t r = __reduce_or_sync(kFull, lane < kSampleWarps ? s_u[lane] : 0u);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t* s_u) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_max_sync(kFull, v);
  if (lane == 0) s_u[warp] = v;
  __syncthreads();
  uint32_t r = __reduce_max_sync(kFull, lane < kSampleWarps ? s_u[lane] : 0u);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t* s_u) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(kFull, v);
  if (lane == 0) s_u[warp] = v;
  __syncthreads();
  uint32_t r = __reduce_add_sync(kFull, lane < kSampleWarps ? s_u[lane] : 0u);
  __syncthreads();
  return r;
}

// Id of the n-th (0-based) id of the row, in increasing id order, for which pred(i) holds,
// or -1. Threads own contiguous id ranges; a block scan of their counts finds the owner.
template <class Pred>
__device__ int64_t block_nth_id(int64_t V, int64_t n, Pred pred, double* s_red,
                                long long* s_found) {
  const int64_t chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int64_t lo = min(V, (int64_t)threadIdx.x * chunk), hi = min(V, lo + chunk);
  int64_t cnt = 0;
  for (int64_t i = lo; i < hi; ++i) cnt += pred(i) ? 1 : 0;
  double total;
  const int64_t before = (int64_t)block_exclusive_scan_d((double)cnt, s_red, &total);
  if (threadIdx.x == 0) *s_found = -1;
  __syncthreads();
  if (n >= before && n < before + cnt) {
    int64_t k = before;
    for (int64_t i = lo; i < hi; ++i) {
      if (pred(i)) {
        if (k == n) {
          *s_found = i;
          break;
        }
        ++k;
      }
    }
  }
  __syncthreads();
  const int64_t r = *s_found;
  __syncthreads();
  return r;
}

template <int DT>
__global__ void __launch_bounds__(kSampleThreads) masked_sample_kernel(const SampleParams p) {
  __shared__ double s_mass[kSampleBins];
  __shared__ uint32_t s_count[kSampleBins];
  __shared__ double s_red[kSampleWarps];
  __shared__ uint32_t s_u[kSampleWarps];
  __shared__ uint32_t s_bin;
  __shared__ double s_above;
  __shared__ long long s_found;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t V = p.vocab;
  using St = typename Elem<DT>::storage;
  const void* rowp = static_cast<const St*>(p.logits) + row * p.row_stride;
  const uint32_t* mrow = p.mask ? p.mask + row * p.mask_stride : nullptr;

  // 1. support: any valid id, NaN, +inf count, the largest finite value (as an order code)
  uint32_t any = 0u, nan = 0u, pinf = 0u, maxo = 0u;
  for (int64_t i = tid; i < V; i += kSampleThreads) {
    if (!sample_valid(mrow, i)) continue;
    any = 1u;
    const float v = sample_value<DT>(rowp, i);
    if (v != v) {
      nan = 1u;
    } else if (v == INFINITY) {
      ++pinf;
    } else if (v != -INFINITY) {
      maxo = max(maxo, ord32(v));
    }
  }
  any = block_or_u32(any, s_u);
  nan = block_or_u32(nan, s_u);
  pinf = block_sum_u32(pinf, s_u);
  maxo = block_max_u32(maxo, s_u);
  const uint32_t status = !any ? kStatusEmptyMask
                          : nan ? kStatusNanInSupport
                          : (!pinf && !maxo) ? kStatusAllNegInf : 0u;
  if (status) {
    if (tid == 0) {
      p.out_idx[row] = -1;
      p.out_status[row] = status;
    }
    return;
  }
  const double u = philox_uniform(p.seed, p.call, (uint32_t)row);

  if (pinf) {
    // 2a. the +inf ids share the mass equally; ranked (equal probabilities) by id
    __shared__ long long s_pick;
    if (tid == 0) {
      const double w = 1.0 / (double)pinf;
      uint32_t m = pinf;
      double cum = 0.0;
      for (uint32_t j = 1; j <= pinf; ++j) {
        cum += w;
        if (cum >= p.top_p) {
          m = j;
          break;
        }
      }
      double kept_total = 0.0;
      for (uint32_t j = 0; j < m; ++j) kept_total += w;
      const double threshold = u * kept_total;
      uint32_t pick = m - 1;
      cum = 0.0;
      for (uint32_t j = 0; j < m; ++j) {
        cum += w;
        if (threshold < cum) {
          pick = j;
          break;
        }
      }
      s_pick = pick;
    }
    __syncthreads();
    const int64_t pick = s_pick;
    const int64_t id = block_nth_id(
        V, pick,
        [&](int64_t i) { return sample_valid(mrow, i) && sample_value<DT>(rowp, i) == INFINITY; },
        s_red, &s_found);
    if (tid == 0) {
      p.out_idx[row] = (int32_t)id;
      p.out_status[row] = 0u;
    }
    return;
  }

  // 2b. finite values: weight exp((v - max) / T), zero weights drop out
  const double vmax = (double)__uint_as_float((maxo & 0x80000000u) ? (maxo & 0x7FFFFFFFu) : ~maxo);
  // divide by T, as the reference does: multiplying by 1/T rounds differently
  auto weight_exact = [&](float v) { return exp(((double)v - vmax) / p.temperature); };

  // 3. total mass and the first radix level (order-code bits 31..21) in one pass
  for (int b = tid; b < kSampleBins; b += kSampleThreads) {
    s_mass[b] = 0.0;
    s_count[b] = 0u;
  }
  __syncthreads();
  double tsum = 0.0;
  for (int64_t i = tid; i < V; i += kSampleThreads) {
    if (!sample_valid(mrow, i)) continue;
    const float v = sample_value<DT>(rowp, i);
    if (v == -INFINITY) continue;
    const double w = weight_exact(v);
    if (!(w > 0.0)) continue;
    tsum += w;
    const uint32_t b = ord32(v) >> 21;
    atomicAdd(&s_mass[b], w);
    atomicAdd(&s_count[b], 1u);
  }
  const double total = block_sum_d(tsum, s_red);

  // 4. levels: find the bin where the probability mass ranked above reaches top_p
  double above = 0.0;  // probability of every token ranked above the current prefix
  uint32_t prefix = 0u;
#pragma unroll
  for (int level = 0; level < 3; ++level) {
    const int shift = level == 0 ? 21 : level == 1 ? 10 : 0;
    const int width = level == 2 ? 10 : 11;
    const int nb = 1 << width;
    if (level > 0) {
      for (int b = tid; b < kSampleBins; b += kSampleThreads) {
        s_mass[b] = 0.0;
        s_count[b] = 0u;
      }
      __syncthreads();
      const int pshift = level == 1 ? 21 : 10;
      for (int64_t i = tid; i < V; i += kSampleThreads) {
        if (!sample_valid(mrow, i)) continue;
        const float v = sample_value<DT>(rowp, i);
        if (v == -INFINITY) continue;
        const uint32_t o = ord32(v);
        if ((o >> pshift) != prefix) continue;
        const double w = weight_exact(v);
        if (!(w > 0.0)) continue;
        const uint32_t b = (o >> shift) & (uint32_t)(nb - 1);
        atomicAdd(&s_mass[b], w);
        atomicAdd(&s_count[b], 1u);
      }
      __syncthreads();
    }
    // thread t owns bins nb-1-2t and nb-2-2t: a scan in descending bin order
    const int b_hi = nb - 1 - 2 * tid, b_lo = b_hi - 1;
    const double p_hi = b_hi >= 0 ? s_mass[b_hi] / total : 0.0;
    const double p_lo = b_lo >= 0 ? s_mass[b_lo] / total : 0.0;
    double sum_all;
    const double before = above + block_exclusive_scan_d(p_hi + p_lo, s_red, &sum_all);
    if (tid == 0) s_bin = 0xFFFFFFFFu;
    __syncthreads();
    if (b_hi >= 0 && s_count[b_hi] && before < p.top_p && before + p_hi >= p.top_p) {
      s_bin = (uint32_t)b_hi;
      s_above = before;
    } else if (b_lo >= 0 && s_count[b_lo] && before + p_hi < p.top_p &&
               before + p_hi + p_lo >= p.top_p) {
      s_bin = (uint32_t)b_lo;
      s_above = before + p_hi;
    }
    __syncthreads();
    if (s_bin == 0xFFFFFFFFu) {
      // the mass never reaches top_p (rounding, or top_p = 1): every token of this prefix
      // is kept; go down into its lowest nonempty bin
      int mine = -1;
      if (b_lo >= 0 && s_count[b_lo]) {
        mine = b_lo;
      } else if (b_hi >= 0 && s_count[b_hi]) {
        mine = b_hi;
      }
      const uint32_t key = mine >= 0 ? (0x80000000u | (uint32_t)(nb - mine)) : 0u;
      const uint32_t best = block_max_u32(key, s_u);
      if (mine >= 0 && (best & 0x7FFFFFFFu) == (uint32_t)(nb - mine)) {
        s_bin = (uint32_t)mine;
        s_above = mine == b_lo ? before + p_hi : before;
      }
      __syncthreads();
    }
    const uint32_t bin = s_bin;
    above = s_above;
    prefix = (prefix << width) | bin;
    __syncthreads();
  }
  // prefix is now the exact order code v* of the value the cut falls on; s_count[bin] of
  // the last level counts its ties
  const uint32_t vstar = prefix;
  const uint32_t ties = s_count[vstar & 1023u];
  const float vstar_f = __uint_as_float((vstar & 0x80000000u) ? (vstar & 0x7FFFFFFFu) : ~vstar);
  const double pstar = weight_exact(vstar_f) / total;
  __shared__ long long s_take;
  if (tid == 0) {
    double cum = above;
    uint32_t take = ties;
    for (uint32_t j = 1; j <= ties; ++j) {
      cum += pstar;
      if (cum >= p.top_p) {
        take = j;
        break;
      }
    }
    s_take = take;
  }
  __syncthreads();
  const int64_t take = s_take;
  // the last kept tie, in id order
  const int64_t last_tie = block_nth_id(
      V, take - 1,
      [&](int64_t i) {
        return sample_valid(mrow, i) && ord32(sample_value<DT>(rowp, i)) == vstar;
      },
      s_red, &s_found);

  // 5. the draw: walk the kept ids (ranked at or above the last kept tie) in id order
  auto kept = [&](int64_t i, double* pi) -> bool {
    if (!sample_valid(mrow, i)) return false;
    const float v = sample_value<DT>(rowp, i);
    if (v == -INFINITY) return false;
    const uint32_t o = ord32(v);
    if (o < vstar || (o == vstar && i > last_tie)) return false;
    *pi = weight_exact(v) / total;
    return true;
  };
  const int64_t chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int64_t lo = min(V, (int64_t)tid * chunk), hi = min(V, lo + chunk);
  double local = 0.0;
  long long last_kept = -1;
  for (int64_t i = lo; i < hi; ++i) {
    double pi;
    if (kept(i, &pi)) {
      local += pi;
      last_kept = i;
    }
  }
  double kept_total;
  const double before = block_exclusive_scan_d(local, s_red, &kept_total);
  const double threshold = u * kept_total;
  __shared__ unsigned long long s_pick_id;
  if (tid == 0) s_pick_id = ~0ull;
  __syncthreads();
  if (last_kept >= 0 && before <= threshold && threshold < before + local) {
    long long pick = last_kept;  // rounding kept the crossing from showing: the chunk's last
    double c = before;
    for (int64_t i = lo; i < hi; ++i) {
      double pi;
      if (kept(i, &pi)) {
        c += pi;
        if (threshold < c) {
          pick = i;
          break;
        }
      }
    }
    atomicMin(&s_pick_id, (unsigned long long)pick);
  }
  __syncthreads();
  unsigned long long id = s_pick_id;
  if (id == ~0ull) {
    // the draw lies past the sum (rounding): the last kept id, as the reference returns
    const uint32_t key = last_kept >= 0 ? (uint32_t)last_kept + 1u : 0u;
    id = (unsigned long long)block_max_u32(key, s_u) - 1ull;
  }
  if (tid == 0) {
    p.out_idx[row] = (int32_t)id;
    p.out_status[row] = 0u;
  }
}
