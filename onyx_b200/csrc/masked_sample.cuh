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

// Element loops with kSampleUnroll independent loads in flight per thread (the value and its
// mask word are loaded side by side). f(i, v) sees the valid ids only.
constexpr int kSampleUnroll = 8;

template <int DT, class F>
__device__ __forceinline__ void for_each_strided(const void* rowp, const uint32_t* mrow,
                                                 int64_t V, F f, bool vec) {
  int64_t start = 0;
  if (vec) {
    // 16-byte vectors: E elements per lane per load, E mask bits from one word (vector
    // starts are multiples of E, so the E bits never straddle two words)
    constexpr int E = 16 / (int)sizeof(typename Elem<DT>::storage);
    const int64_t nvec = V / E;
    const uint4* vp = static_cast<const uint4*>(rowp);
    for (int64_t b = threadIdx.x; b < nvec; b += (int64_t)kSampleThreads * 2) {
      uint4 x[2];
      uint32_t bits[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t vi = b + (int64_t)k * kSampleThreads;
        const bool in = vi < nvec;
        x[k] = in ? __ldg(vp + vi) : make_uint4(0u, 0u, 0u, 0u);
        const int64_t e = vi * E;
        bits[k] = !in ? 0u : !mrow ? 0xFFu : (__ldg(mrow + (e >> 5)) >> (e & 31)) & ((1u << E) - 1u);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t e = (b + (int64_t)k * kSampleThreads) * E;
        const uint32_t w[4] = {x[k].x, x[k].y, x[k].z, x[k].w};
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if (!((bits[k] >> j) & 1u)) continue;
          float v;
          if constexpr (DT == kF32) {
            v = __uint_as_float(w[j]);
          } else {
            const uint32_t h = (w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
            v = DT == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
          }
          f(e + j, v);
        }
      }
    }
    start = nvec * E;
  }
  for (int64_t base = start + threadIdx.x; base < V;
       base += (int64_t)kSampleThreads * kSampleUnroll) {
    float v[kSampleUnroll];
    bool ok[kSampleUnroll];
#pragma unroll
    for (int k = 0; k < kSampleUnroll; ++k) {
      const int64_t i = base + (int64_t)k * kSampleThreads;
      const bool in = i < V;
      v[k] = in ? sample_value<DT>(rowp, i) : 0.f;
      ok[k] = in && sample_valid(mrow, i);
    }
#pragma unroll
    for (int k = 0; k < kSampleUnroll; ++k)
      if (ok[k]) f(base + (int64_t)k * kSampleThreads, v[k]);
  }
}

// The valid ids of [lo, hi) in increasing order; f(i, v) returns true to stop.
template <int DT, class F>
__device__ __forceinline__ void for_each_in_range(const void* rowp, const uint32_t* mrow,
                                                  int64_t lo, int64_t hi, F f) {
  for (int64_t base = lo; base < hi; base += kSampleUnroll) {
    float v[kSampleUnroll];
    bool ok[kSampleUnroll];
#pragma unroll
    for (int k = 0; k < kSampleUnroll; ++k) {
      const int64_t i = base + k;
      const bool in = i < hi;
      v[k] = in ? sample_value<DT>(rowp, i) : 0.f;
      ok[k] = in && sample_valid(mrow, i);
    }
#pragma unroll
    for (int k = 0; k < kSampleUnroll; ++k)
      if (ok[k] && f(base + k, v[k])) return;
  }
}

// Warp-range iteration with compaction: warp w owns the contiguous ids [w R, (w + 1) R)
// (R a multiple of 8). In steps of 256 ids (8 per lane, one 16-byte load for 16-bit types
// when the row is aligned), the ids that pred(i, v) keeps are packed, in id order, into the
// warp's shared-memory buffer and handed to batch(has, i, v) 32 at a time, one per lane, so
// that the per-id work (a float64 exp) runs on full warps however sparse the kept ids are.
// batch is called by every lane of the warp (has = this lane holds an id) and may use warp
// collectives; it returns true (warp-uniformly) to stop the walk.
constexpr int kSampleStep = 256;  // ids per warp step: 8 per lane

struct WarpBuf {
  float v[kSampleStep];
  uint16_t off[kSampleStep];  // id - step base
};

template <int DT, class Pred, class Batch>
__device__ __forceinline__ void warp_range_batches(const void* rowp, const uint32_t* mrow,
                                                   int64_t lo, int64_t hi, bool vec,
                                                   WarpBuf* buf, Pred pred, Batch batch) {
  using St = typename Elem<DT>::storage;
  const int lane = threadIdx.x & 31;
  for (int64_t base = lo; base < hi; base += kSampleStep) {
    const int64_t e0 = base + 8 * lane;
    float v[8];
    uint32_t keep = 0u;
    const uint32_t word = e0 < hi && mrow ? __ldg(mrow + (e0 >> 5)) >> (e0 & 31) : 0xFFu;
    if (vec && e0 + 8 <= hi) {
      if constexpr (DT == kF32) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const St*>(rowp) + e0));
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(static_cast<const St*>(rowp) + e0) + 1);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(w[j]);
      } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const St*>(rowp) + e0));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t h = (w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
          v[j] = DT == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = e0 + j < hi ? sample_value<DT>(rowp, e0 + j) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (e0 + j < hi && ((word >> j) & 1u) && pred(e0 + j, v[j])) keep |= 1u << j;
    // pack the kept ids in id order (lane-major, then j)
    const uint32_t cnt = __popc(keep);
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += n;
    }
    const uint32_t total = __shfl_sync(kFull, incl, 31);
    uint32_t pos = incl - cnt;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if ((keep >> j) & 1u) {
        buf->v[pos] = v[j];
        buf->off[pos] = (uint16_t)(8 * lane + j);
        ++pos;
      }
    }
    __syncwarp();
    bool stop = false;
    for (uint32_t k = 0; k < total && !stop; k += 32) {
      const bool has = k + lane < total;
      stop = batch(has, has ? base + buf->off[k + lane] : (int64_t)-1,
                   has ? buf->v[k + lane] : 0.f);  // warp-uniform
    }
    __syncwarp();
    if (stop) return;
  }
}

// Id of the n-th (0-based) id of the row, in increasing id order, for which pred(i) holds,
// or -1. Threads own contiguous id ranges; a block scan of their counts finds the owner.
template <int DT, class Pred>
__device__ int64_t block_nth_id(const void* rowp, const uint32_t* mrow, int64_t V, int64_t n,
                                Pred pred, double* s_red, long long* s_found) {
  const int64_t chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int64_t lo = min(V, (int64_t)threadIdx.x * chunk), hi = min(V, lo + chunk);
  int64_t cnt = 0;
  for_each_in_range<DT>(rowp, mrow, lo, hi, [&](int64_t i, float v) {
    cnt += pred(i, v) ? 1 : 0;
    return false;
  });
  double total;
  const int64_t before = (int64_t)block_exclusive_scan_d((double)cnt, s_red, &total);
  if (threadIdx.x == 0) *s_found = -1;
  __syncthreads();
  if (n >= before && n < before + cnt) {
    int64_t k = before;
    for_each_in_range<DT>(rowp, mrow, lo, hi, [&](int64_t i, float v) {
      if (!pred(i, v)) return false;
      if (k == n) {
        *s_found = i;
        return true;
      }
      ++k;
      return false;
    });
  }
  __syncthreads();
  const int64_t r = *s_found;
  __syncthreads();
  return r;
}

// dynamic shared memory: the warps' compaction buffers, reused for the histograms
constexpr size_t kSampleSmemBytes = sizeof(WarpBuf) * kSampleWarps;
static_assert(kSampleSmemBytes >= kSampleBins * (sizeof(double) + sizeof(uint32_t)), "");

template <int DT>
__global__ void __launch_bounds__(kSampleThreads) masked_sample_kernel(const SampleParams p) {
  extern __shared__ __align__(16) unsigned char s_dyn[];
  WarpBuf* const s_bufs = reinterpret_cast<WarpBuf*>(s_dyn);
  double* const s_mass = reinterpret_cast<double*>(s_dyn);
  uint32_t* const s_count = reinterpret_cast<uint32_t*>(s_dyn + kSampleBins * sizeof(double));
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
  const bool vec = ((uintptr_t)rowp & 15u) == 0;  // 16-byte loads (block-uniform)

  // 1. support: any valid id, NaN, +inf count, the largest finite value (as an order code)
  uint32_t any = 0u, nan = 0u, pinf = 0u, maxo = 0u;
  for_each_strided<DT>(rowp, mrow, V, [&](int64_t, float v) {
    any = 1u;
    if (v != v) {
      nan = 1u;
    } else if (v == INFINITY) {
      ++pinf;
    } else if (v != -INFINITY) {
      maxo = max(maxo, ord32(v));
    }
  }, vec);
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
    const int64_t id = block_nth_id<DT>(
        rowp, mrow, V, pick, [&](int64_t, float v) { return v == INFINITY; }, s_red, &s_found);
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

  // 3. total mass and the number of weighted ids
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t wrange = ((V + 31) / 32 + 7) / 8 * 8;  // each warp's ids, a multiple of 8
  const int64_t wlo = min(V, (int64_t)warp * wrange), whi = min(V, wlo + wrange);
  double tsum = 0.0;
  uint32_t nw = 0u;
  warp_range_batches<DT>(
      rowp, mrow, wlo, whi, vec, &s_bufs[warp], [&](int64_t, float v) { return v != -INFINITY; },
      [&](bool has, int64_t, float v) {
        if (has) {
          const double w = weight_exact(v);
          if (w > 0.0) {
            tsum += w;
            ++nw;
          }
        }
        return false;
      });
  __syncthreads();  // the buffers become the histograms
  const double total = block_sum_d(tsum, s_red);
  nw = block_sum_u32(nw, s_u);
  // The first radix level only needs the ids that can hold the cut: those of weight below
  // tau = (1 - top_p) total / (2 nw) weigh at most (1 - top_p) total / 2 together, so the
  // ids above tau reach top_p by themselves. (This keeps the shared-memory histogram from
  // taking one atomic per id of the row, most of them on a few hot bins.)
  const double tau = (1.0 - p.top_p) * total / (2.0 * (double)nw);
  // the same cut on the value, tested before any exp: w >= tau iff v >= max + T ln(tau)
  const double vtau = tau > 0.0 ? vmax + p.temperature * log(tau) : -INFINITY;

  // 4. levels: find the bin where the probability mass ranked above reaches top_p. With
  //    top_p = 1 every weighted id is kept: no cut to find.
  double above = 0.0;  // probability of every token ranked above the current prefix
  uint32_t prefix = 0u;
  const bool keep_all = !(p.top_p < 1.0);
#pragma unroll
  for (int level = 0; level < 3; ++level) {
    if (keep_all) break;  // block-uniform
    const int shift = level == 0 ? 21 : level == 1 ? 10 : 0;
    const int width = level == 2 ? 10 : 11;
    const int nb = 1 << width;
    for (int b = tid; b < kSampleBins; b += kSampleThreads) {
      s_mass[b] = 0.0;
      s_count[b] = 0u;
    }
    __syncthreads();
    const int pshift = level == 1 ? 21 : 10;  // the previous level's shift (unused at level 0)
    for_each_strided<DT>(rowp, mrow, V, [&](int64_t, float v) {
      if (v == -INFINITY) return;
      const uint32_t o = ord32(v);
      if (level > 0 && (o >> pshift) != prefix) return;
      if (level == 0 && (double)v < vtau) return;
      const double w = weight_exact(v);
      if (!(w > 0.0)) return;
      const uint32_t b = (o >> shift) & (uint32_t)(nb - 1);
      atomicAdd(&s_mass[b], w);
      atomicAdd(&s_count[b], 1u);
    }, vec);
    __syncthreads();
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
  const uint32_t vstar = keep_all ? 0u : prefix;  // 0: below every value's code
  const uint32_t ties = keep_all ? 0u : s_count[vstar & 1023u];
  const float vstar_f = __uint_as_float((vstar & 0x80000000u) ? (vstar & 0x7FFFFFFFu) : ~vstar);
  const double pstar = keep_all ? 0.0 : weight_exact(vstar_f) / total;
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
  const int64_t last_tie =
      keep_all ? V
               : block_nth_id<DT>(
                     rowp, mrow, V, take - 1, [&](int64_t, float v) { return ord32(v) == vstar; },
                     s_red, &s_found);

  // 5. the draw: walk the kept ids (ranked at or above the last kept tie) in id order
  auto kept = [&](int64_t i, float v) {
    if (v == -INFINITY) return false;
    const uint32_t o = ord32(v);
    return o > vstar || (o == vstar && i <= last_tie);
  };
  __syncthreads();  // the histograms become the buffers again
  double wsum = 0.0;       // this warp's kept mass (same in every lane)
  uint32_t wlast = 0u;     // 1 + the warp's last kept id of positive probability, or 0
  warp_range_batches<DT>(rowp, mrow, wlo, whi, vec, &s_bufs[warp], kept,
                         [&](bool has, int64_t i, float v) {
                           const double pi = has ? weight_exact(v) / total : 0.0;
                           wsum += warp_sum_d(pi);
                           wlast = max(wlast, __reduce_max_sync(
                                                  kFull, pi > 0.0 ? (uint32_t)i + 1u : 0u));
                           return false;
                         });
  // warp sums in warp order = id order: every warp gets its exclusive prefix and the total
  __shared__ double s_wsum[kSampleWarps];
  if (lane == 0) s_wsum[warp] = wsum;
  __syncthreads();
  double pre = s_wsum[lane], incl = pre;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  double excl = __shfl_up_sync(kFull, incl, 1);
  if (lane == 0) excl = 0.0;
  const double kept_total = __shfl_sync(kFull, incl, 31);
  const double before = __shfl_sync(kFull, excl, warp);
  (void)pre;
  const double threshold = u * kept_total;
  __shared__ unsigned long long s_pick_id;
  if (tid == 0) s_pick_id = ~0ull;
  __syncthreads();
  if (wlast && before <= threshold && threshold < before + wsum) {
    // this warp's range holds the crossing: walk it again with running sums
    double cum = before;
    unsigned long long pick = (unsigned long long)wlast - 1ull;  // if rounding hides it
    warp_range_batches<DT>(rowp, mrow, wlo, whi, vec, &s_bufs[warp], kept,
                           [&](bool has, int64_t i, float v) {
                             const double pi = has ? weight_exact(v) / total : 0.0;
                             double run = pi;
#pragma unroll
                             for (int o = 1; o < 32; o <<= 1) {
                               const double n = __shfl_up_sync(kFull, run, o);
                               if (lane >= o) run += n;
                             }
                             const unsigned hit =
                                 __ballot_sync(kFull, has && pi > 0.0 && threshold < cum + run);
                             if (hit) {
                               pick = (unsigned long long)__shfl_sync(kFull, i, __ffs(hit) - 1);
                               return true;
                             }
                             cum += __shfl_sync(kFull, run, 31);
                             return false;
                           });
    if (lane == 0) atomicMin(&s_pick_id, pick);
  }
  __syncthreads();
  unsigned long long id = s_pick_id;
  if (id == ~0ull) {
    // the draw lies past the sum (rounding): the last kept id, as the reference returns
    id = (unsigned long long)block_max_u32(wlast, s_u) - 1ull;
  }
  if (tid == 0) {
    p.out_idx[row] = (int32_t)id;
    p.out_status[row] = 0u;
  }
}
