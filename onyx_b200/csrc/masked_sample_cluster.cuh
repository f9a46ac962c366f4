// Masked temperature / top-p sampling, cluster form (included by masked_select.cu after
// masked_sample.cuh, inside namespace onyx). Same distribution, top-p set and draw as
// masked_sample_kernel (the reference's _filtered_reference_weights, selection.py:103-150,
// and the Philox4x32-10 draw); a different decomposition:
//
// * One cluster of k CTAs (k = 1..16) per row. CTA r copies ids [r S, min(V, (r + 1) S)) of
//   the row, values and mask words, into its shared memory once (cp.async; from an aligned
//   row each warp copies its own range in groups and starts on the first group to land).
//   Every later pass reads shared memory, so a row costs one HBM read and the passes run on
//   k SMs at once.
// * Cluster-wide sums and decisions: each CTA stores its block result into every CTA's box
//   for its rank (distributed shared memory), the cluster barrier publishes the boxes, and
//   every CTA combines the k boxes from its own shared memory in rank order. All CTAs therefore
//   hold bit-identical totals and take the same branches (the cluster barriers always match
//   up).
// * bf16 rows with a mask: each warp lists its valid ids from the mask words, and the later
//   passes run over the lists. The cut comes from a per-value table (one bin per bf16 value
//   of the row's top 16 exponents, each sign): counts per bin, one exp per nonempty bin, a
//   block scan over the bins in value order (see "per-value table" below). The radix select
//   that follows serves the other dtypes, and bf16 rows whose cut falls outside the table.
// * The top-p cut by radix select. Candidates are the ids of weight at least tau = (1 - top_p) total / (2 n)
//   (the ids below it weigh at most (1 - top_p) total / 2 together, so the ids above reach
//   top_p by themselves); in value terms v >= vtau = max + T ln(tau). All candidate order
//   codes lie between code(vtau) and code(max), so they share the leading bits of those
//   two codes: the radix select starts below that common prefix, which spreads the
//   candidates over the bins instead of piling them on the few bins of one exponent. It
//   stops at the last bit a 16-bit source type can set (bit 16 for bf16, 13 for f16; the
//   lower bits of the code follow from the sign), where each bin is one exact value: the
//   last level counts ids per value and its mass is count x weight(value), one exp per
//   bin. Earlier levels (wide ranges, f32) add per-id weights.
// * The draw. Per warp (warps own contiguous id ranges; CTA ranks follow id order): the
//   probability of the kept ids ranked strictly above the cut value, and the count of ids
//   equal to it (the ties, kept in id order up to the count the cut needs). One exchange
//   gives every CTA the kept mass before each CTA; the last warp, in id order, whose kept
//   mass starts at or below u x kept_total walks its range with running sums and writes the
//   sampled id.
// Sums over many tokens are tree reductions, so their rounding differs from the reference's
// sequential sums by a few units in the last place, as in masked_sample_kernel.

constexpr int kCsThreads = 1024;
constexpr int kCsWarps = kCsThreads / 32;
constexpr int kCsMaxCluster = 16;
constexpr int kCsBins = 2048;   // widest radix level (11 bits)
constexpr int kCsSliceAlign = 256;  // ids per slice are a multiple of this (8 per lane x 32)
constexpr int kCsStageGroups = 4;   // copy groups per warp when staging an aligned row

struct ClusterSampleParams {
  const void* logits;
  int64_t row_stride;  // elements
  int64_t vocab;
  const uint32_t* mask;  // nullptr: every id valid
  int64_t mask_stride;   // words
  double temperature;
  double top_p;
  unsigned long long seed;
  unsigned long long call;
  int32_t* out_idx;
  uint32_t* out_status;
  int32_t k;      // CTAs per row (the cluster size)
  int32_t slice;  // ids per CTA, a multiple of kCsSliceAlign
  // dynamic shared memory carve-up (byte offsets)
  int32_t off_words;  // staged mask words
  int32_t off_work;   // warp compaction buffers / local histogram
  int32_t off_comb;   // this CTA's slice of the combined histogram
};

// One mailbox per exchange; two, used alternately, so that a CTA may post the next
// exchange while another still reads the previous one (a barrier separates them).
struct CsMail {
  double d[2];
  uint32_t u[4];
};

struct CsCut {  // a crossing of the per-value table scan
  double above;   // probability ranked above the cut value
  double p;       // probability of one id of the cut value
  uint32_t ties;  // ids of the cut value
  uint32_t take;  // of those, kept (in id order)
};

struct CsHist {  // local histogram of one radix level (overlays the compaction buffers)
  double mass[kCsBins];
  uint32_t count[kCsBins];
};

__device__ __forceinline__ void cs_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cs_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// generic address of the same shared-memory object in CTA `rank` of the cluster
template <class T>
__device__ __forceinline__ T* cs_remote_mut(T* p, uint32_t rank) {
  unsigned long long out;
  asm("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(p), "r"(rank));
  return reinterpret_cast<T*>(out);
}

template <class T>
__device__ __forceinline__ const T* cs_remote(const T* p, uint32_t rank) {
  unsigned long long out;
  asm("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(p), "r"(rank));
  return reinterpret_cast<const T*>(out);
}

__device__ __forceinline__ void cs_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cs_cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cs_cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void cs_cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// waits until at most n (0..4) of this thread's committed copy groups are still pending
__device__ __forceinline__ void cs_cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
  }
}

// Eight staged ids of one lane, from slice-relative id j0 (a multiple of 8): their values
// and the bits of those that are valid and below lim (lim <= the slice's id count, so
// j0 < lim keeps all eight reads inside the staged buffer, whose length is a multiple of 8).
template <int DT>
__device__ __forceinline__ uint32_t cs_load8(const unsigned char* vals, const uint32_t* words,
                                             int j0, int lim, float v[8]) {
  if (j0 >= lim) {
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = 0.f;
    return 0u;
  }
  if constexpr (DT == kF32) {
    const uint4 a = *reinterpret_cast<const uint4*>(vals + (size_t)j0 * 4);
    const uint4 b = *reinterpret_cast<const uint4*>(vals + (size_t)j0 * 4 + 16);
    v[0] = __uint_as_float(a.x);
    v[1] = __uint_as_float(a.y);
    v[2] = __uint_as_float(a.z);
    v[3] = __uint_as_float(a.w);
    v[4] = __uint_as_float(b.x);
    v[5] = __uint_as_float(b.y);
    v[6] = __uint_as_float(b.z);
    v[7] = __uint_as_float(b.w);
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(vals + (size_t)j0 * 2);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const uint32_t h = (w[t >> 1] >> (16 * (t & 1))) & 0xFFFFu;
      v[t] = DT == kBF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
    }
  }
  uint32_t m = words ? (words[j0 >> 5] >> (j0 & 31)) & 0xFFu : 0xFFu;
  const int left = lim - j0;
  if (left < 8) m &= left > 0 ? (1u << left) - 1u : 0u;
  return m;
}

// Warp-range walk over staged ids [lo, hi) (slice-relative, lo a multiple of 8) with
// compaction: in steps of 256 ids (8 per lane), keep8(j0, v, m) -- called by every lane of
// the warp, so it may use warp collectives -- returns the bits of the lane's 8 ids to keep;
// the kept ids are packed in id order into the warp's buffer and handed to
// batch(has, j, x) 32 at a time, one per lane (the per-id work runs on full warps however
// sparse the kept ids are). batch is called by every lane and returns true, warp-uniformly,
// to stop the walk.
template <int DT, class Keep8, class Batch>
__device__ __forceinline__ void cs_warp_batches(const unsigned char* vals, const uint32_t* words,
                                                int lo, int hi, WarpBuf* buf, Keep8 keep8,
                                                Batch batch) {
  const int lane = threadIdx.x & 31;
  for (int s = lo; s < hi; s += kSampleStep) {
    const int j0 = s + 8 * lane;
    float v[8];
    const uint32_t m = cs_load8<DT>(vals, words, j0, hi, v);
    const uint32_t keep = keep8(j0, v, m);
    if (!__any_sync(kFull, keep != 0u)) continue;  // nothing kept in this step
    const uint32_t cnt = __popc(keep);
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t total = __shfl_sync(kFull, incl, 31);
    uint32_t pos = incl - cnt;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if ((keep >> t) & 1u) {
        buf->v[pos] = v[t];
        buf->off[pos] = (uint16_t)(8 * lane + t);
        ++pos;
      }
    }
    __syncwarp();
    bool stop = false;
    for (uint32_t q = 0; q < total && !stop; q += 32) {
      const bool has = q + lane < total;
      stop = batch(has, has ? s + (int)buf->off[q + lane] : -1, has ? buf->v[q + lane] : 0.f);
    }
    __syncwarp();
    if (stop) return;
  }
}

__device__ __forceinline__ float cs_code_to_float(uint32_t code) {
  return __uint_as_float((code & 0x80000000u) ? (code & 0x7FFFFFFFu) : ~code);
}

// The full 32-bit order code from its bits [rb, 32): below bit rb a 16-bit source value has
// zero bits, which the code keeps for a non-negative value and inverts for a negative one.
template <int RB>
__device__ __forceinline__ uint32_t cs_full_code(uint32_t hi_bits) {
  if constexpr (RB == 0) {
    return hi_bits;
  } else {
    const uint32_t c = hi_bits << RB;
    return (c & 0x80000000u) ? c : (c | ((1u << RB) - 1u));
  }
}

// position of the (r+1)-th set bit of an 8-bit mask (r < popc(m))
__device__ __forceinline__ int cs_nth_bit8(uint32_t m, uint32_t r) {
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if ((m >> t) & 1u) {
      if (r == 0u) return t;
      --r;
    }
  }
  return 7;
}

// ---- per-value table (bf16) -------------------------------------------------------------
// A bf16 weight exp((v - max) / T) depends only on the 16-bit value, and a row's values
// cluster in a few binary exponents. The table has one bin per value whose exponent field lies
// in the kVtExps exponents below and at the row's largest finite one, for each sign, in
// descending value order: bins [0, kVtHalf) the positive values from the largest down,
// [kVtHalf, kVtBins) the negative ones from the smallest magnitude down. Zeros and magnitudes
// below the table form the "small" region, which lies between the two halves in value order;
// its ids keep a per-id weight.
constexpr int kVtExps = 16;
constexpr int kVtHalf = kVtExps * 128;
constexpr int kVtBins = 2 * kVtHalf;
static_assert(kVtBins * (sizeof(double) + sizeof(uint32_t)) <= sizeof(WarpBuf) * kCsWarps,
              "the per-value table overlays the compaction buffers");
// Each warp lists the offsets of its valid ids in id order (written by the support pass), so
// the count, kept-mass and draw passes touch valid ids only. A warp with more valid ids than
// a list holds walks its whole range instead.
constexpr int kVtListCap = kVtBins * (int)sizeof(double) / (int)sizeof(uint16_t) / kCsWarps;
// bf16 work area: the id lists, then the local counts (until the bin sums), over which the
// probabilities of the lookup table are stored (the whole table with top_p = 1)
constexpr int kVtListBytes = kVtListCap * kCsWarps * (int)sizeof(uint16_t);
constexpr int kVtMinKeepAllSlice = 16384;  // with top_p = 1, smaller slices take exp per id
constexpr int kVtWorkBytes = kVtListBytes + kVtBins * (int)sizeof(double);
static_assert(kVtWorkBytes >= (int)(sizeof(WarpBuf) * kCsWarps) &&
              kVtWorkBytes >= kVtListBytes + kVtBins * (int)sizeof(uint32_t), "bf16 work area");
constexpr uint32_t kNoList = 0xFFFFFFFFu;

// largest exponent field among the valid (bit set in `bits`), finite bf16 values of a vector
// of eight; 0 if none
__device__ __forceinline__ uint32_t vt_max_exponent(const uint4& a, uint32_t bits) {
  uint32_t m01, m23, m45, m67;
  expand8_16(bits, m01, m23, m45, m67);
  const uint32_t w[4] = {a.x & m01, a.y & m23, a.z & m45, a.w & m67};
  uint32_t best = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t e = (w[i] >> 7) & 0x00FF00FFu;  // both halves' exponent fields
    e &= ~__vcmpeq2(e, 0x00FF00FFu);          // infinities and NaN are not finite
    best = __vmaxu2(best, e);
  }
  return max(best & 0xFFFFu, best >> 16);
}

// table bin of a finite bf16 bit pattern h, or -1 for the small region
__device__ __forceinline__ int vt_bin(uint32_t h, int e_top) {
  if ((h & 0x7FFFu) == 0u) return -1;  // +-0
  const int de = e_top - (int)((h >> 7) & 0xFFu);
  if (de < 0 || de >= kVtExps) return -1;  // (de < 0: an infinity, never weighted here)
  const int m = (int)(h & 0x7Fu);
  return (h & 0x8000u) ? kVtHalf + (kVtExps - 1 - de) * 128 + m : de * 128 + (127 - m);
}

// the bf16 value of table bin b (a NaN for a bin below exponent 0, which holds no value)
__device__ __forceinline__ float vt_value(int b, int e_top) {
  const bool neg = b >= kVtHalf;
  const int r = neg ? b - kVtHalf : b;
  const int de = neg ? kVtExps - 1 - (r >> 7) : (r >> 7);
  const int m = neg ? (r & 127) : 127 - (r & 127);
  const int e = e_top - de;
  if (e < 0) return __int_as_float(0x7FC00000);
  return bf16_bits_to_f32((neg ? 0x8000u : 0u) | ((uint32_t)e << 7) | (uint32_t)m);
}

// bins of the combined area per row (split over the cluster): the radix levels' widest level,
// or for bf16 the per-value table
__host__ __device__ constexpr int cs_comb_bins(int dt) { return dt == kBF16 ? kVtBins : kCsBins; }

// bins per CTA of the combined area: a share of cs_comb_bins(dt) over k CTAs, rounded up to
// a multiple of 4 so that four consecutive bins always have one owner and sit 16-byte
// aligned in its area (vector reads across the cluster)
__host__ __device__ constexpr int cs_comb_share(int dt, int k) {
  return ((cs_comb_bins(dt) + k - 1) / k + 3) / 4 * 4;
}

template <int DT>
__global__ void __launch_bounds__(kCsThreads, 1)
    masked_sample_cluster_kernel(const ClusterSampleParams p) {
  using St = typename Elem<DT>::storage;
  constexpr int kElem = (int)sizeof(St);
  constexpr int kRb = DT == kBF16 ? 16 : DT == kF16 ? 13 : 0;  // lowest bit a value can set
  extern __shared__ __align__(16) unsigned char s_dyn[];
  __shared__ CsMail s_box[2][kCsMaxCluster];  // per exchange parity: every CTA's mailbox
  __shared__ double s_red[kSampleWarps];
  __shared__ uint32_t s_u[kSampleWarps];
  __shared__ double s_wmass[kCsWarps];    // per warp: total weight, then kept mass above the cut
  __shared__ uint32_t s_wcount[kCsWarps];  // per warp: +inf ids, then ties of the cut value
  __shared__ uint32_t s_wexp[kCsWarps];    // per warp: largest finite exponent field (bf16)
  __shared__ uint32_t s_bin, s_ties;
  __shared__ CsCut s_cut[kCsWarps];        // per warp: its earliest crossing of the table scan
  __shared__ uint32_t s_cutrank[kCsWarps];
  __shared__ uint32_t s_lcount[kCsWarps];  // per warp: listed ids, kNoList when not listed
  __shared__ double s_above;
  __shared__ long long s_take;
  __shared__ int s_walk_warp;
  __shared__ double s_walk_before;
  __shared__ long long s_walk_rank;

  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");  // (see exchange)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = p.k;
  const uint32_t rank = cs_rank();
  const int64_t row = blockIdx.x / k;
  const int64_t V = p.vocab;
  const int64_t lo = (int64_t)rank * p.slice;
  const int n = (int)max((int64_t)0, min((int64_t)p.slice, V - lo));
  unsigned char* const s_vals = s_dyn;
  uint32_t* const s_words = p.mask ? reinterpret_cast<uint32_t*>(s_dyn + p.off_words) : nullptr;
  WarpBuf* const s_bufs = reinterpret_cast<WarpBuf*>(s_dyn + p.off_work);
  CsHist* const s_hist = reinterpret_cast<CsHist*>(s_dyn + p.off_work);
  const int comb_cap = cs_comb_share(DT, k);
  double* const s_comb_p = reinterpret_cast<double*>(s_dyn + p.off_comb);
  uint32_t* const s_comb_c =
      reinterpret_cast<uint32_t*>(s_dyn + p.off_comb + ((comb_cap * 8 + 15) & ~15));

  // warp w owns the contiguous staged ids [wlo, whi): whole mask words (32 ids each)
  const int wrange = ((n + 31) / 32 + 31) / 32 * 32;
  const int wlo = min(n, warp * wrange), whi = min(n, wlo + wrange);
  // this warp's mask words [wlo / 32, wq1): none for an empty range (wlo = n need not be a
  // multiple of 32, and the word holding id n - 1 belongs to the warp before)
  const int wq1 = whi > wlo ? (whi + 31) >> 5 : wlo >> 5;
  const int wsteps = (whi - wlo + kSampleStep - 1) / kSampleStep;
  const int spg = (wsteps + kCsStageGroups - 1) / kCsStageGroups;  // steps per copy group

  // 0. stage this CTA's ids, values and mask words. From a 16-byte aligned row every warp
  //    copies its own range: one group of mask words, then kCsStageGroups groups of values,
  //    so the support pass starts on the first groups while the others are in flight; otherwise
  //    every thread copies element by element and the block waits for the whole slice.
  const St* const g = static_cast<const St*>(p.logits) + row * p.row_stride + lo;
  const bool warp_staged = ((uintptr_t)g & 15u) == 0;
  if (warp_staged) {
    if (p.mask) {
      const uint32_t* gm = p.mask + row * p.mask_stride + (lo >> 5);
      for (int q = (wlo >> 5) + lane; q < wq1; q += 32) cs_cp_async4(s_words + q, gm + q);
    }
    cs_cp_async_commit();
    for (int gi = 0; gi < kCsStageGroups; ++gi) {
      const int i1 = min(wsteps, (gi + 1) * spg);
      for (int i = gi * spg; i < i1; ++i) {
        const int j0 = wlo + i * kSampleStep + 8 * lane;
        if (j0 + 8 <= whi) {
#pragma unroll
          for (int c = 0; c < kElem / 2; ++c)
            cs_cp_async16(s_vals + (size_t)j0 * kElem + 16 * c,
                          reinterpret_cast<const unsigned char*>(g + j0) + 16 * c);
        } else {
          for (int j = j0; j < whi; ++j) reinterpret_cast<St*>(s_vals)[j] = __ldg(g + j);
        }
      }
      cs_cp_async_commit();
    }
  } else {
    for (int j = tid; j < n; j += kCsThreads) reinterpret_cast<St*>(s_vals)[j] = __ldg(g + j);
    if (p.mask) {
      const uint32_t* gm = p.mask + row * p.mask_stride + (lo >> 5);
      const int nw = (n + 31) >> 5;
      for (int q = tid; q < nw; q += kCsThreads) cs_cp_async4(s_words + q, gm + q);
    }
    cs_cp_async_wait_all();
    __syncthreads();
  }

  // Exchange: thread q stores this CTA's mailbox into CTA q's box for this rank, then the
  // cluster barrier (release / acquire) publishes every box; after it a CTA reads only its own
  // shared memory, so no CTA ever reads another's after the last exchange. Boxes alternate by
  // parity: a CTA stores into a box again only after the next barrier, which every CTA
  // reaches after its last read of that box.
  int slot = 0;
  const CsMail* s_all = s_box[0];
  bool first_exchange = true;
  auto exchange = [&](const CsMail& mine) {
    // the first store into another CTA waits for the barrier phase every CTA arrived at when
    // it started: then every CTA of the cluster is running
    if (first_exchange) {
      asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
      first_exchange = false;
    }
    if (tid < k) *cs_remote_mut(&s_box[slot][rank], (uint32_t)tid) = mine;
    cs_cluster_sync();
    s_all = s_box[slot];
    slot ^= 1;
  };

  // 1. support: the masked, NaN-propagating maximum; any valid id at all; for bf16 the
  //    largest finite exponent. bf16 rows with a mask first list each warp's
  //    valid ids, in id order, from its mask words alone (they land first), then take the
  //    support from the listed ids as their copy groups land. Other rows, and warps with
  //    more valid ids than a list holds, read every id (packed pairs for 16-bit types).
  const bool listing = DT == kBF16 && s_words != nullptr;
  uint16_t* const s_list = reinterpret_cast<uint16_t*>(s_dyn + p.off_work) + warp * kVtListCap;
  const uint16_t* const s_h = reinterpret_cast<const uint16_t*>(s_vals);
  uint32_t lcount = 0u;  // this warp's valid ids (warp-uniform); listed while <= kVtListCap
  uint32_t any = 0u, lcode = 0u, lexp = 0u;
  bool listed_support = false;
  if (listing) {
    if (warp_staged) {
      cs_cp_async_wait_pending(kCsStageGroups);  // the mask words (the first group)
      __syncwarp();
    }
    for (int qb = wlo >> 5; qb < wq1; qb += 32) {  // warp-uniform: one word per lane
      const int q = qb + lane;
      uint32_t bits = 0u;
      if (q < wq1) {
        bits = s_words[q];
        const int left = whi - 32 * q;
        if (left < 32) bits &= (1u << left) - 1u;
      }
      const uint32_t c = __popc(bits);
      uint32_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
      }
      const uint32_t tot = __shfl_sync(kFull, incl, 31);
      if (lcount + tot <= (uint32_t)kVtListCap) {
        uint32_t pos = lcount + incl - c;
        for (uint32_t mm = bits; mm; mm &= mm - 1u)
          s_list[pos++] = (uint16_t)(32 * q - wlo + __ffs(mm) - 1);
      }
      lcount += tot;
    }
    if (lcount <= (uint32_t)kVtListCap) {
      __syncwarp();  // the list is visible to the whole warp
      float lmax = -INFINITY;
      int landed = 0;  // value groups known to have landed
      for (uint32_t i0 = 0; i0 < lcount; i0 += 32) {  // warp-uniform
        if (warp_staged) {
          // the group of the last id of these 32 (the list is in id order)
          const int need = (int)(s_list[min(lcount - 1u, i0 + 31u)] / kSampleStep) / spg + 1;
          if (need > landed) {
            cs_cp_async_wait_pending(kCsStageGroups - need);
            __syncwarp();
            landed = need;
          }
        }
        const uint32_t i = i0 + lane;
        if (i < lcount) {
          const uint32_t h = s_h[wlo + s_list[i]];
          lmax = max_nan_f32(lmax, bf16_bits_to_f32(h));
          const uint32_t e = (h >> 7) & 0xFFu;
          if (e != 0xFFu) lexp = max(lexp, e);
        }
      }
      any = lcount ? 1u : 0u;
      lcode = ord32(lmax);  // NaN: the largest code
      listed_support = true;
    }
  }
  if (lane == 0) s_lcount[warp] = listed_support ? lcount : kNoList;  // (read by this warp)
  if (!listed_support) {
    float lmax = -INFINITY;
    uint32_t pm = 0u;
    if constexpr (DT != kF32) pm = Packed16<DT>::kNegInfPair;
    int staged_to = 0, next_group = 0;  // steps [0, staged_to) of this warp have landed
    for (int s = wlo; s < whi; s += kSampleStep) {  // warp-uniform
      if (warp_staged && (s - wlo) / kSampleStep >= staged_to) {
        cs_cp_async_wait_pending(kCsStageGroups - 1 - next_group);
        __syncwarp();  // every lane's copies of the group are visible to the warp
        ++next_group;
        staged_to += spg;
      }
      const int j0 = s + 8 * lane;
      if (j0 >= whi) continue;
      uint32_t m = s_words ? (s_words[j0 >> 5] >> (j0 & 31)) & 0xFFu : 0xFFu;
      const int left = whi - j0;
      if (left < 8) m &= (1u << left) - 1u;
      any |= m;
      if constexpr (DT == kF32) {
        const uint4 a = *reinterpret_cast<const uint4*>(s_vals + (size_t)j0 * 4);
        const uint4 b = *reinterpret_cast<const uint4*>(s_vals + (size_t)j0 * 4 + 16);
        lmax = max_nan_f32(lmax, max_nan_f32(Vec16<kF32>::masked_max(a, m & 0xFu),
                                             Vec16<kF32>::masked_max(b, m >> 4)));
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(s_vals + (size_t)j0 * 2);
        pm = Packed16<DT>::pmax(pm, Packed16<DT>::masked_pair_max(a, m));
        if constexpr (DT == kBF16) lexp = max(lexp, vt_max_exponent(a, m));
      }
    }
    if constexpr (DT != kF32) lmax = Packed16<DT>::pair_to_f32_max(pm);
    lcode = ord32(lmax);  // NaN: the largest code
  }
  {
    const uint32_t wa = __reduce_or_sync(kFull, any), wc = __reduce_max_sync(kFull, lcode);
    const uint32_t we = __reduce_max_sync(kFull, lexp);
    if (lane == 0) {
      s_wcount[warp] = wa;
      s_u[warp] = wc;
      s_wexp[warp] = we;
    }
    __syncthreads();
    CsMail m = {};
    m.u[0] = __reduce_or_sync(kFull, s_wcount[lane]);
    m.u[1] = __reduce_max_sync(kFull, s_u[lane]);
    m.u[2] = __reduce_max_sync(kFull, s_wexp[lane]);
    exchange(m);  // (its barriers also end every read of s_wcount and s_u)
  }
  uint32_t c_any = 0u, c_code = 0u, c_exp = 0u;
  for (int q = 0; q < k; ++q) {
    c_any |= s_all[q].u[0];
    c_code = max(c_code, s_all[q].u[1]);
    c_exp = max(c_exp, s_all[q].u[2]);
  }
  constexpr uint32_t kOrd32PosInf = 0xFF800000u;
  const uint32_t status = !c_any ? kStatusEmptyMask
                          : c_code == kOrd32NaN ? kStatusNanInSupport
                          : c_code == kOrd32NegInf ? kStatusAllNegInf : 0u;
  const uint32_t c_maxo = c_code;  // the largest finite value when status == 0 and no +inf
  const double u = philox_uniform(p.seed, p.call, (uint32_t)row);

  if (status) {
    if (rank == 0 && tid == 0) {
      p.out_idx[row] = -1;
      p.out_status[row] = status;
    }
  } else if (c_code == kOrd32PosInf) {
    // 2a. the +inf ids share the mass equally; ranked (equal probabilities) by id. Count
    //     them per warp and per CTA.
    uint32_t pinf = 0u;
    for (int s = wlo; s < whi; s += kSampleStep) {
      float v[8];
      const uint32_t m = cs_load8<DT>(s_vals, s_words, s + 8 * lane, whi, v);
#pragma unroll
      for (int t = 0; t < 8; ++t) pinf += (((m >> t) & 1u) && v[t] == INFINITY) ? 1u : 0u;
    }
    {
      const uint32_t wp = __reduce_add_sync(kFull, pinf);
      if (lane == 0) s_wcount[warp] = wp;
    }
    __syncthreads();
    pinf = __reduce_add_sync(kFull, s_wcount[lane]);
    {
      CsMail m = {};
      m.u[0] = pinf;
      exchange(m);
    }
    uint32_t c_pinf = 0u, pinf_before = 0u;
    for (int q = 0; q < k; ++q) {
      if (q < (int)rank) pinf_before += s_all[q].u[0];
      c_pinf += s_all[q].u[0];
    }
    if (tid == 0) {
      const double w = 1.0 / (double)c_pinf;
      uint32_t m = c_pinf;
      double cum = 0.0;
      for (uint32_t j = 1; j <= c_pinf; ++j) {
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
      s_take = pick;
      // the warp of this CTA holding the pick, if any
      s_walk_warp = -1;
      if (pick >= pinf_before && pick < pinf_before + pinf) {
        uint32_t before = pinf_before;
        for (int w2 = 0; w2 < kCsWarps; ++w2) {
          if (pick < before + s_wcount[w2]) {
            s_walk_warp = w2;
            s_walk_rank = (long long)(pick - before);
            break;
          }
          before += s_wcount[w2];
        }
      }
    }
    __syncthreads();
    if (warp == s_walk_warp) {
      uint32_t r = (uint32_t)s_walk_rank;  // the pick among this warp's +inf ids
      for (int s = wlo; s < whi; s += kSampleStep) {
        float v[8];
        const int j0 = s + 8 * lane;
        const uint32_t m = cs_load8<DT>(s_vals, s_words, j0, whi, v);
        uint32_t inf_bits = 0u;
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (((m >> t) & 1u) && v[t] == INFINITY) inf_bits |= 1u << t;
        const uint32_t c = __popc(inf_bits);
        uint32_t incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += t;
        }
        const uint32_t tot = __shfl_sync(kFull, incl, 31);
        if (r < tot) {
          if (r >= incl - c && r < incl) {
            p.out_idx[row] = (int32_t)(lo + j0 + cs_nth_bit8(inf_bits, r - (incl - c)));
            p.out_status[row] = 0u;
          }
          break;
        }
        r -= tot;
      }
    }
  } else {
    // 2b. finite values: weight exp((v - max) / T), zero weights drop out
    const double vmax = (double)cs_code_to_float(c_maxo);
    // divide by T, as the reference does: multiplying by 1/T rounds differently
    auto weight_exact = [&](float x) { return exp(((double)x - vmax) / p.temperature); };

    const bool keep_all = !(p.top_p < 1.0);
    double total = 0.0;
    uint32_t nwt = 0u;
    uint32_t vstar = 0u;  // order code of the cut value (0: below every value: keep all)
    uint32_t ties = 0u;
    double above = 0.0;  // probability of every id ranked above the current prefix
    bool have_cut = keep_all;  // the cut is known (nothing to cut with top_p = 1)
    // bf16: the per-value table. Steps 5 and 6 look a kept id's probability up when its bin
    // is below lut_bins: every bin with top_p = 1, the kCsThreads largest positive values
    // otherwise
    // the table serves bf16 rows, except with top_p = 1 on small slices, where one exp per
    // valid id costs less than the table's cluster barriers and reads
    const bool vt = DT == kBF16 && !(keep_all && p.slice <= kVtMinKeepAllSlice);
    const int lut_bins = vt ? (keep_all ? kVtBins : kCsThreads) : 0;
    int cut_warp = -1;  // the table scan's crossing (s_cut) also gives pstar and take; -2:
                        // nothing is cut (top_p = 1)
    const int e_top = (int)c_exp;
    // the lookup table: one probability per bin, over the local counts once they are summed
    double* const s_lut = reinterpret_cast<double*>(s_dyn + p.off_work + kVtListBytes);
    uint32_t* const s_tc = reinterpret_cast<uint32_t*>(s_dyn + p.off_work + kVtListBytes);
    if (vt) {
      // 3t. this CTA's counts per bin (into the count half of the work area) and the per-id
      //     weights of its small-region ids
      for (int b = tid; b < kVtBins; b += kCsThreads) s_tc[b] = 0u;
      __syncthreads();
      double fsum = 0.0;
      uint32_t fn = 0u;
      auto count_small = [&](uint32_t h) {
        const double w = weight_exact(bf16_bits_to_f32(h));
        if (w > 0.0) {
          fsum += w;
          ++fn;
        }
      };
      const uint32_t ln = s_lcount[warp];
      if (ln != kNoList) {
        for (uint32_t i = lane; i < ln; i += 32) {
          const uint32_t h = s_h[wlo + s_list[i]];
          if (h == 0xFF80u) continue;  // -inf: weight 0
          const int b = vt_bin(h, e_top);
          if (b >= 0)
            atomicAdd(&s_tc[b], 1u);
          else
            count_small(h);
        }
      } else {
        for (int s = wlo; s < whi; s += kSampleStep) {
          float v[8];
          const uint32_t m = cs_load8<DT>(s_vals, s_words, s + 8 * lane, whi, v);
          uint32_t small = 0u;  // this lane's ids of the small region among its eight
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if (!((m >> t) & 1u) || v[t] == -INFINITY) continue;
            const int b = vt_bin(__float_as_uint(v[t]) >> 16, e_top);
            if (b >= 0)
              atomicAdd(&s_tc[b], 1u);
            else
              small |= 1u << t;
          }
          for (; small; small &= small - 1u)  // rare: zeros and tiny magnitudes
            count_small(s_h[s + 8 * lane + __ffs(small) - 1]);
        }
      }
      cs_cluster_sync();  // every CTA's counts are complete
      // 3u. this CTA's share of the bins: counts summed over the cluster in rank order, one
      //     exp per nonempty bin; zero weights drop out
      const int per = comb_cap;
      const int b0 = (int)rank * per, b1 = min(kVtBins, b0 + per);
      double smass = 0.0;
      uint32_t sn = 0u;
      // (two bins per thread at a time: every remote count read in flight together, and the
      // two exp chains side by side)
      for (int b = b0 + tid; b < b1; b += 2 * kCsThreads) {
        const int b2 = b + kCsThreads;
        const bool two = b2 < b1;
        uint32_t c1 = 0u, c2 = 0u;
#pragma unroll
        for (int q = 0; q < kCsMaxCluster; ++q) {
          if (q < k) {
            const uint32_t* rq = cs_remote(s_tc, (uint32_t)q);
            c1 += rq[b];
            if (two) c2 += rq[b2];
          }
        }
        double w1 = c1 ? weight_exact(vt_value(b, e_top)) : 0.0;
        double w2 = c2 ? weight_exact(vt_value(b2, e_top)) : 0.0;
        if (!(w1 > 0.0)) {
          w1 = 0.0;
          c1 = 0u;
        }
        if (!(w2 > 0.0)) {
          w2 = 0.0;
          c2 = 0u;
        }
        s_comb_p[b - b0] = w1;
        s_comb_c[b - b0] = c1;
        smass += (double)c1 * w1;
        sn += c1;
        if (two) {
          s_comb_p[b2 - b0] = w2;
          s_comb_c[b2 - b0] = c2;
          smass += (double)c2 * w2;
          sn += c2;
        }
      }
      {
        const double wm = warp_sum_d(smass + fsum), wf = warp_sum_d(fsum);
        const uint32_t wn = __reduce_add_sync(kFull, sn + fn);
        if (lane == 0) {
          s_wmass[warp] = wm;
          s_red[warp] = wf;
          s_wcount[warp] = wn;
        }
      }
      __syncthreads();
      {
        double cm = 0.0, cf = 0.0;
        for (int w2 = 0; w2 < kCsWarps; ++w2) {
          cm += s_wmass[w2];
          cf += s_red[w2];
        }
        CsMail m = {};
        m.d[0] = cm;
        m.d[1] = cf;
        m.u[0] = __reduce_add_sync(kFull, s_wcount[lane]);
        exchange(m);  // (its cluster barrier also completes every CTA's share)
      }
      double small_w = 0.0;
      for (int q = 0; q < k; ++q) {
        total += s_all[q].d[0];
        small_w += s_all[q].d[1];
        nwt += s_all[q].u[0];
      }
      // 3v. the bins' probabilities, read from their owners' shares (every remote read of the
      //     local counts ended at the exchange). With top_p = 1 nothing is cut: thread t
      //     stores bins 4t .. 4t+3 for the kept-mass and draw passes. Otherwise 3w finds the
      //     cut, and a kept id's probability is a lookup among the top kCsThreads bins or one
      //     exp.
      static_assert(kVtBins == 4 * kCsThreads && kCsThreads <= kVtHalf, "bins per thread");
      // thread t's four bins 4t .. 4t+3 (one owner for all four: shares are multiples of 4)
      auto load4 = [&](double* pv, uint32_t* cb) {
        const int q = 4 * tid / per, o = 4 * tid - q * per;
        const double2* wq = reinterpret_cast<const double2*>(cs_remote(s_comb_p, (uint32_t)q) + o);
        const double2 w01 = wq[0], w23 = wq[1];
        const uint4 c4 = *reinterpret_cast<const uint4*>(cs_remote(s_comb_c, (uint32_t)q) + o);
        pv[0] = w01.x / total;
        pv[1] = w01.y / total;
        pv[2] = w23.x / total;
        pv[3] = w23.y / total;
        cb[0] = c4.x;
        cb[1] = c4.y;
        cb[2] = c4.z;
        cb[3] = c4.w;
      };
      // the earliest crossing over the block (rank 2b for bin b, 2 kVtHalf - 1 for the small
      // region; a block-scan rounding could let two threads see one). The crossing thread
      // also counts the ties the cut keeps, adding them one by one as the reference does.
      auto publish_cut = [&](uint32_t mine, double mine_before, uint32_t mine_ties,
                             double mine_p) {
        const uint32_t wmin = __reduce_min_sync(kFull, mine);
        if (mine != 0xFFFFFFFFu && mine == wmin && !(mine & 1u)) {
          double c2 = mine_before;
          uint32_t take = mine_ties;
          for (uint32_t j = 1; j <= mine_ties; ++j) {
            c2 += mine_p;
            if (c2 >= p.top_p) {
              take = j;
              break;
            }
          }
          s_cut[warp] = CsCut{mine_before, mine_p, mine_ties, take};
        }
        if (lane == 0) s_cutrank[warp] = wmin;
        __syncthreads();
        const uint32_t r = s_cutrank[lane];
        const uint32_t cut = __reduce_min_sync(kFull, r);
        if (cut != 0xFFFFFFFFu && !(cut & 1u)) {
          cut_warp = __ffs(__ballot_sync(kFull, r == cut)) - 1;
          have_cut = true;
          vstar = ord32(vt_value((int)(cut >> 1), e_top));
          above = s_cut[cut_warp].above;
          ties = s_cut[cut_warp].ties;
        }
      };
      if (keep_all) {
        double pv[4];
        uint32_t cb[4];
        load4(pv, cb);
#pragma unroll
        for (int i = 0; i < 4; ++i) s_lut[4 * tid + i] = pv[i];
        __syncthreads();
        cut_warp = -2;
      } else {
        // 3w, first stage: the kCsThreads largest positive values' bins, one per thread.
        //     The cut of a top_p < 1 row nearly always lies among them; their probabilities
        //     become the lookup table (in the area of the local counts, which no CTA reads
        //     any more).
        {
          const int b = tid, q = b / per, o = b - q * per;
          const double pvb = cs_remote(s_comb_p, (uint32_t)q)[o] / total;
          const uint32_t c = cs_remote(s_comb_c, (uint32_t)q)[o];
          s_lut[b] = pvb;
          const double pbb = (double)c * pvb;
          double sum_all;
          const double before = block_exclusive_scan_d(pbb, s_red, &sum_all);  // (also orders
          // the lookup table's stores before any read)
          const bool cross = c && before < p.top_p && before + pbb >= p.top_p;
          publish_cut(cross ? 2u * (uint32_t)b : 0xFFFFFFFFu, before, c, pvb);
        }
        if (!have_cut) {
          // second stage: every bin, four per thread, in value order; the small region
          // follows bin kVtHalf - 1
          double pv[4];
          uint32_t cb[4];
          load4(pv, cb);
          const double small_p = small_w / total;
          double tm = 0.0;
#pragma unroll
          for (int i = 0; i < 4; ++i) tm += (double)cb[i] * pv[i];
          const bool small_after = 4 * tid + 3 == kVtHalf - 1;
          if (small_after) tm += small_p;
          double sum_all;
          const double before = block_exclusive_scan_d(tm, s_red, &sum_all);
          double cum = before;
          uint32_t mine = 0xFFFFFFFFu, mine_ties = 0u;
          double mine_before = 0.0, mine_p = 0.0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const double pbi = (double)cb[i] * pv[i];
            if (cb[i] && cum < p.top_p && cum + pbi >= p.top_p && mine == 0xFFFFFFFFu) {
              mine = 2u * (uint32_t)(4 * tid + i);
              mine_before = cum;
              mine_ties = cb[i];
              mine_p = pv[i];
            }
            cum += pbi;
          }
          if (small_after && mine == 0xFFFFFFFFu && small_p > 0.0 && cum < p.top_p &&
              cum + small_p >= p.top_p)
            mine = 2u * kVtHalf - 1u;
          publish_cut(mine, mine_before, mine_ties, mine_p);
        }
      }
      // without a cut here (it falls among the small-region ids, or the sum never reaches
      // top_p) the radix levels below find it; their histograms overwrite the id lists, so
      // only a cut from this scan (cut_warp >= 0), or none needed (-2), leaves them for step 5
    } else {
      // 3. total weight and the number of weighted ids
      double tsum = 0.0;
      uint32_t nw = 0u;
      cs_warp_batches<DT>(
          s_vals, s_words, wlo, whi, &s_bufs[warp],
          [&](int, const float* v, uint32_t m) {
            uint32_t keep = 0u;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (((m >> t) & 1u) && v[t] != -INFINITY) keep |= 1u << t;
            return keep;
          },
          [&](bool has, int, float x) {
            if (has) {
              const double w = weight_exact(x);
              if (w > 0.0) {
                tsum += w;
                ++nw;
              }
            }
            return false;
          });
      {
        const double wt = warp_sum_d(tsum);
        const uint32_t wn = __reduce_add_sync(kFull, nw);
        if (lane == 0) {
          s_wmass[warp] = wt;
          s_wcount[warp] = wn;
        }
      }
      __syncthreads();
      {
        double ct = 0.0;
        for (int w2 = 0; w2 < kCsWarps; ++w2) ct += s_wmass[w2];
        CsMail m = {};
        m.d[0] = ct;
        m.u[0] = __reduce_add_sync(kFull, s_wcount[lane]);
        exchange(m);
      }
      for (int q = 0; q < k; ++q) {
        total += s_all[q].d[0];
        nwt += s_all[q].u[0];
      }
    }
    // 4. radix levels from below the candidates' common prefix down to one exact value
    if (!have_cut) {
      // candidates: weight >= tau = (1 - top_p) total / (2 n), i.e. value >= vtau; as a
      // float test, x >= fthr with fthr the least float not below vtau
      const double tau = (1.0 - p.top_p) * total / (2.0 * (double)nwt);
      const double vtau = tau > 0.0 ? vmax + p.temperature * log(tau) : -INFINITY;
      float fthr = (float)vtau;
      if ((double)fthr < vtau) fthr = nextafterf(fthr, INFINITY);
      const uint32_t lowc = fthr == -INFINITY ? kOrd32NegInf + 1u : min(ord32(fthr), c_maxo);
      const uint32_t diff = lowc ^ c_maxo;
      int top = diff ? 32 - __clz(diff) : 0;  // bits [top, 32) are the same in every candidate
      if (top < kRb + 1) top = kRb + 1;
      uint32_t prefix = top >= 32 ? 0u : (c_maxo >> top);
      int cur = top;
      while (cur > kRb) {  // cluster-uniform
        const int width = min(11, cur - kRb);
        const int shift = cur - width;
        const int nb = 1 << width;
        const bool final_level = shift == kRb;
        for (int b = tid; b < nb; b += kCsThreads) {
          s_hist->mass[b] = 0.0;
          s_hist->count[b] = 0u;
        }
        __syncthreads();
        for (int s = wlo; s < whi; s += kSampleStep) {
          float v[8];
          const uint32_t m = cs_load8<DT>(s_vals, s_words, s + 8 * lane, whi, v);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float x = v[t];
            if (!((m >> t) & 1u) || !(x >= fthr) || x == -INFINITY) continue;
            const uint32_t o = ord32(x);
            if (cur < 32 && (o >> cur) != prefix) continue;
            const uint32_t b = (o >> shift) & (uint32_t)(nb - 1);
            if (final_level) {
              atomicAdd(&s_hist->count[b], 1u);
            } else {
              const double w = weight_exact(x);
              if (w > 0.0) {
                atomicAdd(&s_hist->mass[b], w);
                atomicAdd(&s_hist->count[b], 1u);
              }
            }
          }
        }
        cs_cluster_sync();  // every CTA's local histogram is complete
        // this CTA sums its share of the bins over the cluster, in rank order
        const int per = (nb + k - 1) / k;
        const int b0 = (int)rank * per, b1 = min(nb, b0 + per);
        for (int b = b0 + tid; b < b1; b += kCsThreads) {
          // every remote read in flight at once, then the sums in rank order
          uint32_t cq[kCsMaxCluster];
#pragma unroll
          for (int q = 0; q < kCsMaxCluster; ++q)
            cq[q] = q < k ? cs_remote(s_hist, (uint32_t)q)->count[b] : 0u;
          uint32_t csum = 0u;
#pragma unroll
          for (int q = 0; q < kCsMaxCluster; ++q) csum += cq[q];
          double msum = 0.0;
          if (!final_level) {
            double mq[kCsMaxCluster];
#pragma unroll
            for (int q = 0; q < kCsMaxCluster; ++q)
              mq[q] = q < k ? cs_remote(s_hist, (uint32_t)q)->mass[b] : 0.0;
#pragma unroll
            for (int q = 0; q < kCsMaxCluster; ++q) msum += mq[q];
          }
          double pb = 0.0;
          if (final_level) {
            // one exact value per bin: mass = count x its probability
            if (csum) {
              const double w =
                  weight_exact(cs_code_to_float(cs_full_code<kRb>((prefix << width) | (uint32_t)b)));
              if (w > 0.0) {
                pb = (double)csum * (w / total);
              } else {
                csum = 0u;
              }
            }
          } else {
            pb = msum / total;
          }
          s_comb_p[b - b0] = pb;
          s_comb_c[b - b0] = csum;
        }
        cs_cluster_sync();  // the combined histogram is complete
        // thread t owns bins nb-1-2t and nb-2-2t: a scan in descending bin order
        const int b_hi = nb - 1 - 2 * tid, b_lo = b_hi - 1;
        double p_hi = 0.0, p_lo = 0.0;
        uint32_t c_hi = 0u, c_lo = 0u;
        if (b_hi >= 0) {
          const int q = b_hi / per, o = b_hi - q * per;
          p_hi = cs_remote(s_comb_p, (uint32_t)q)[o];
          c_hi = cs_remote(s_comb_c, (uint32_t)q)[o];
        }
        if (b_lo >= 0) {
          const int q = b_lo / per, o = b_lo - q * per;
          p_lo = cs_remote(s_comb_p, (uint32_t)q)[o];
          c_lo = cs_remote(s_comb_c, (uint32_t)q)[o];
        }
        double sum_all;
        const double before = above + block_exclusive_scan_d(p_hi + p_lo, s_red, &sum_all);
        if (tid == 0) s_bin = 0xFFFFFFFFu;
        __syncthreads();
        if (c_hi && before < p.top_p && before + p_hi >= p.top_p) {
          s_bin = (uint32_t)b_hi;
          s_above = before;
          s_ties = c_hi;
        } else if (c_lo && before + p_hi < p.top_p && before + p_hi + p_lo >= p.top_p) {
          s_bin = (uint32_t)b_lo;
          s_above = before + p_hi;
          s_ties = c_lo;
        }
        __syncthreads();
        if (s_bin == 0xFFFFFFFFu) {
          // the mass never reaches top_p (rounding): every id of this prefix is kept; go
          // down into its lowest nonempty bin
          int mine = -1;
          if (c_lo) {
            mine = b_lo;
          } else if (c_hi) {
            mine = b_hi;
          }
          const uint32_t key = mine >= 0 ? (0x80000000u | (uint32_t)(nb - mine)) : 0u;
          const uint32_t best = block_max_u32(key, s_u);
          if (mine >= 0 && (best & 0x7FFFFFFFu) == (uint32_t)(nb - mine)) {
            s_bin = (uint32_t)mine;
            s_above = mine == b_lo ? before + p_hi : before;
            s_ties = mine == b_lo ? c_lo : c_hi;
          }
          __syncthreads();
        }
        prefix = (prefix << width) | s_bin;
        above = s_above;
        ties = s_ties;
        cur = shift;
        __syncthreads();
      }
      vstar = cs_full_code<kRb>(prefix);
    }
    // the ties: ids equal to the cut value, kept in id order while the cumulative sum, added
    // one by one as the reference does, stays below top_p
    // as a float: ord32 order is float order with -0 == +0, and no value here is NaN; with
    // every weighted id kept, -inf is the bound (above it: every finite value)
    const float vstar_f = keep_all ? -INFINITY : cs_code_to_float(vstar);
    double pstar = 0.0;
    uint32_t take = 0u;
    if (cut_warp >= 0) {  // (block-uniform)
      pstar = s_cut[cut_warp].p;
      take = s_cut[cut_warp].take;
    } else if (cut_warp == -1) {
      pstar = keep_all ? 0.0 : weight_exact(vstar_f) / total;
      if (tid == 0) {
        double cum = above;
        uint32_t tk = ties;
        for (uint32_t j = 1; j <= ties; ++j) {
          cum += pstar;
          if (cum >= p.top_p) {
            tk = j;
            break;
          }
        }
        s_take = tk;
      }
      __syncthreads();  // (also: every warp is done with the histogram before the buffers)
      take = (uint32_t)s_take;
    }

    // probability of one kept id: the table's entry for its value, or exp per id
    auto prob = [&](float x) -> double {
      if (lut_bins) {
        const int b = vt_bin(__float_as_uint(x) >> 16, e_top);
        if (b >= 0 && b < lut_bins) return s_lut[b];  // the whole table, or its top
      }
      return weight_exact(x) / total;
    };

    // 5. per warp: probability of the ids ranked above the cut value, and the ties
    double wabove = 0.0;
    uint32_t wties = 0u;
    if (vt) {
      // (the per-value path keeps no per-warp totals and no compaction buffers: one pass of
      // lookups, ids of the small region weighted one by one)
      double acc = 0.0;
      uint32_t lane_ties = 0u;
      const uint32_t ln = cut_warp != -1 ? s_lcount[warp] : kNoList;
      if (ln != kNoList) {
        for (uint32_t i = lane; i < ln; i += 32) {
          const float x = bf16_bits_to_f32(s_h[wlo + s_list[i]]);
          if (x > vstar_f)
            acc += prob(x);
          else if (!keep_all && x == vstar_f)
            ++lane_ties;
        }
      } else {
        for (int s = wlo; s < whi; s += kSampleStep) {
          float v[8];
          const uint32_t m = cs_load8<DT>(s_vals, s_words, s + 8 * lane, whi, v);
          uint32_t kept = 0u;
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if (!((m >> t) & 1u)) continue;
            if (v[t] > vstar_f)
              kept |= 1u << t;
            else if (!keep_all && v[t] == vstar_f)
              ++lane_ties;
          }
          for (; kept; kept &= kept - 1u) {
            const int t = __ffs(kept) - 1;
            acc += prob(bf16_bits_to_f32(
                reinterpret_cast<const uint16_t*>(s_vals)[s + 8 * lane + t]));
          }
        }
      }
      wabove = warp_sum_d(acc);
      wties = __reduce_add_sync(kFull, lane_ties);
    } else if (keep_all) {
      wabove = s_wmass[warp] / total;
    } else {
      uint32_t lane_ties = 0u;
      cs_warp_batches<DT>(
          s_vals, s_words, wlo, whi, &s_bufs[warp],
          [&](int, const float* v, uint32_t m) {
            uint32_t keep = 0u;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              if (!((m >> t) & 1u)) continue;
              if (v[t] > vstar_f) keep |= 1u << t;
              if (v[t] == vstar_f) ++lane_ties;
            }
            return keep;
          },
          [&](bool has, int, float x) {
            wabove += warp_sum_d(has ? weight_exact(x) / total : 0.0);
            return false;
          });
      wties = __reduce_add_sync(kFull, lane_ties);
    }
    __syncthreads();  // every warp has read s_wmass
    if (lane == 0) {
      s_wmass[warp] = wabove;
      s_wcount[warp] = wties;
    }
    __syncthreads();
    {
      double ca = 0.0;
      uint32_t ct = 0u;
      for (int w2 = 0; w2 < kCsWarps; ++w2) {
        ca += s_wmass[w2];
        ct += s_wcount[w2];
      }
      CsMail m = {};
      m.d[0] = ca;
      m.u[0] = ct;
      exchange(m);
    }
    // kept mass per CTA: above the cut plus its share of the first `take` ties
    double kept_total = 0.0;
    {
      uint32_t tb = 0u;
      for (int q = 0; q < k; ++q) {
        const uint32_t tq = s_all[q].u[0];
        const uint32_t mq = take > tb ? min(take - tb, tq) : 0u;
        kept_total += s_all[q].d[0] + (double)mq * pstar;
        tb += tq;
      }
    }
    const double threshold = u * kept_total;
    // the walk belongs to the last CTA, then the last warp, in id order whose kept mass is
    // positive and starts at or below the threshold (warp 0 scans: lane q holds CTA q, then
    // lane w holds warp w)
    if (warp == 0) {
      auto excl_u = [&](uint32_t x) {
        uint32_t incl = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += t;
        }
        return incl - x;
      };
      auto excl_d = [&](double x) {
        double incl = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double t = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += t;
        }
        const double e = __shfl_up_sync(kFull, incl, 1);
        return lane == 0 ? 0.0 : e;
      };
      const uint32_t tq = lane < k ? s_all[lane].u[0] : 0u;
      const uint32_t tbq = excl_u(tq);
      const uint32_t mq = take > tbq ? min(take - tbq, tq) : 0u;
      const double kq = lane < k ? s_all[lane].d[0] + (double)mq * pstar : 0.0;
      const double kbq = excl_d(kq);
      const unsigned cq = __ballot_sync(kFull, kq > 0.0 && kbq <= threshold);
      const int chosen = cq ? 31 - __clz(cq) : -1;
      int walk = -1;
      double walk_before = 0.0;
      uint32_t walk_rank = 0u;
      if (chosen == (int)rank) {
        const double cbefore = __shfl_sync(kFull, kbq, chosen);
        const uint32_t cties = __shfl_sync(kFull, tbq, chosen);
        const uint32_t tw = s_wcount[lane];
        const uint32_t tbw = cties + excl_u(tw);
        const uint32_t mw = take > tbw ? min(take - tbw, tw) : 0u;
        const double kw = s_wmass[lane] + (double)mw * pstar;
        const double kbw = cbefore + excl_d(kw);
        const unsigned cw = __ballot_sync(kFull, kw > 0.0 && kbw <= threshold);
        if (cw) {
          walk = 31 - __clz(cw);
          walk_before = __shfl_sync(kFull, kbw, walk);
          walk_rank = __shfl_sync(kFull, tbw, walk);
        }
      }
      if (lane == 0) {
        s_walk_warp = walk;
        s_walk_before = walk_before;
        s_walk_rank = walk_rank;
      }
    }
    __syncthreads();
    const uint32_t walk_list = vt && cut_warp != -1 && warp == s_walk_warp
                                   ? s_lcount[warp] : kNoList;
    if (walk_list != kNoList) {
      // 6. the draw from this warp's list: 32 valid ids at a time, one per lane, in id order;
      //    running sums by a warp scan
      double cum = s_walk_before;
      uint32_t tie_rank = (uint32_t)s_walk_rank;  // ties of the cut value before these ids
      int pick = -1, last = -1;  // slice-relative
      for (uint32_t i0 = 0; i0 < walk_list && pick < 0; i0 += 32) {  // warp-uniform
        const uint32_t i = i0 + lane;
        int j = -1;
        float x = -INFINITY;
        if (i < walk_list) {
          j = wlo + s_list[i];
          x = bf16_bits_to_f32(s_h[j]);
        }
        const bool tie = !keep_all && x == vstar_f;
        const unsigned tb = __ballot_sync(kFull, tie);
        const uint32_t r = tie_rank + __popc(tb & ((1u << lane) - 1u));
        tie_rank += __popc(tb);
        const bool keep = x > vstar_f || (tie && r < take);
        const double pi = keep ? prob(x) : 0.0;
        double run = pi;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double t = __shfl_up_sync(kFull, run, o);
          if (lane >= o) run += t;
        }
        const int lastj = (int)__reduce_max_sync(kFull, pi > 0.0 ? (uint32_t)(j + 1) : 0u);
        if (lastj) last = lastj - 1;
        const unsigned hit = __ballot_sync(kFull, pi > 0.0 && threshold < cum + run);
        if (hit) pick = __shfl_sync(kFull, j, __ffs(hit) - 1);
        cum += __shfl_sync(kFull, run, 31);
      }
      if (pick < 0) pick = last;  // the draw lies past this warp's sum (rounding)
      if (lane == 0) {
        p.out_idx[row] = (int32_t)(lo + pick);
        p.out_status[row] = 0u;
      }
    } else if (warp == s_walk_warp && vt) {
      // 6. the draw: walk this warp's kept ids in id order with running sums; one step of
      //    256 ids at a time, each lane's eight in id order after the lanes before it
      double cum = s_walk_before;
      uint32_t tie_rank = (uint32_t)s_walk_rank;  // ties of the cut value before this step
      int pick = -1, last = -1;  // slice-relative
      for (int s = wlo; s < whi && pick < 0; s += kSampleStep) {  // warp-uniform
        const int j0 = s + 8 * lane;
        float v[8];
        const uint32_t m = cs_load8<DT>(s_vals, s_words, j0, whi, v);
        uint32_t above_bits = 0u, tie_bits = 0u;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (!((m >> t) & 1u)) continue;
          if (v[t] > vstar_f) above_bits |= 1u << t;
          if (!keep_all && v[t] == vstar_f) tie_bits |= 1u << t;
        }
        const uint32_t c = __popc(tie_bits);
        uint32_t incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += t;
        }
        uint32_t r = tie_rank + incl - c;
        tie_rank += __shfl_sync(kFull, incl, 31);
        uint32_t keep = above_bits;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if ((tie_bits >> t) & 1u) {
            if (r < take) keep |= 1u << t;
            ++r;
          }
        }
        double pl[8];
        double lsum = 0.0;
        int llast = -1;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          pl[t] = ((keep >> t) & 1u) ? prob(v[t]) : 0.0;
          lsum += pl[t];
          if (pl[t] > 0.0) llast = j0 + t;
        }
        double run = lsum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double t = __shfl_up_sync(kFull, run, o);
          if (lane >= o) run += t;
        }
        const int sl = (int)__reduce_max_sync(kFull, (uint32_t)(llast + 1)) - 1;
        if (sl >= 0) last = sl;
        const unsigned hit = __ballot_sync(kFull, lsum > 0.0 && threshold < cum + run);
        if (hit) {
          const int wl = __ffs(hit) - 1;
          int pk = -1;
          if (lane == wl) {
            double r2 = cum + (run - lsum);
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              if (pl[t] > 0.0 && pk < 0) {
                r2 += pl[t];
                if (threshold < r2) pk = j0 + t;
              }
            }
            if (pk < 0) pk = llast;  // the running sums round differently from the scan
          }
          pick = __shfl_sync(kFull, pk, wl);
        }
        cum += __shfl_sync(kFull, run, 31);
      }
      if (pick < 0) pick = last;  // the draw lies past this warp's sum (rounding)
      if (lane == 0) {
        p.out_idx[row] = (int32_t)(lo + pick);
        p.out_status[row] = 0u;
      }
    } else if (warp == s_walk_warp) {
      // 6. the draw: walk this warp's kept ids in id order with running sums
      double cum = s_walk_before;
      uint32_t tie_rank = (uint32_t)s_walk_rank;  // ties of the cut value before this step
      int pick = -1, last = -1;  // slice-relative
      cs_warp_batches<DT>(
          s_vals, s_words, wlo, whi, &s_bufs[warp],
          [&](int, const float* v, uint32_t m) {
            uint32_t above_bits = 0u, tie_bits = 0u;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              if (!((m >> t) & 1u)) continue;
              if (v[t] > vstar_f) above_bits |= 1u << t;
              if (v[t] == vstar_f) tie_bits |= 1u << t;
            }
            // ranks of this lane's ties among the row's ties, in id order
            const uint32_t c = __popc(tie_bits);
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t t = __shfl_up_sync(kFull, incl, o);
              if (lane >= o) incl += t;
            }
            uint32_t r = tie_rank + incl - c;
            tie_rank += __shfl_sync(kFull, incl, 31);
            uint32_t keep = above_bits;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              if ((tie_bits >> t) & 1u) {
                if (r < take) keep |= 1u << t;
                ++r;
              }
            }
            return keep;
          },
          [&](bool has, int j, float x) {
            const double pi = has ? weight_exact(x) / total : 0.0;
            double run = pi;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const double t = __shfl_up_sync(kFull, run, o);
              if (lane >= o) run += t;
            }
            const unsigned hit = __ballot_sync(kFull, has && pi > 0.0 && threshold < cum + run);
            const int lastj = __reduce_max_sync(kFull, (has && pi > 0.0) ? (uint32_t)(j + 1) : 0u);
            if (lastj) last = lastj - 1;
            if (hit) {
              pick = __shfl_sync(kFull, j, __ffs(hit) - 1);
              return true;
            }
            cum += __shfl_sync(kFull, run, 31);
            return false;
          });
      if (pick < 0) pick = last;  // the draw lies past this warp's sum (rounding)
      if (lane == 0) {
        p.out_idx[row] = (int32_t)(lo + pick);
        p.out_status[row] = 0u;
      }
    }
  }
  // (no final cluster barrier: every read of another CTA's shared memory precedes the last
  // exchange's barrier)
}
