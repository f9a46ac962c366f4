// Streaming form of the masked selection (included by masked_select.cu inside namespace
// onyx, after the cluster kernel). Same contract as masked_select_kernel and the cluster
// kernel in the argmax (and gather), shard-key and speculative-verify modes; a different
// decomposition, for batches of several waves:
//
// * One CTA per SM for the whole launch. The rows' elements, in row order, are cut into
//   256-element units, and CTA c owns the contiguous units [c T / n, (c + 1) T / n) of the
//   T units of the launch, so every CTA streams the same number of bytes (to one unit).
// * One producer thread per CTA moves its range into a ring of kStreamStages shared-memory
//   stages with plain 1-D bulk copies (cp.async.bulk, global -> this CTA's shared memory,
//   completion counted on the stage's "full" mbarrier). A piece -- at most 32 KB of logits
//   and their mask words, never crossing a row boundary -- fills one stage. Up to
//   kStreamStages pieces are in flight per SM, so DRAM sees a steady queue from the first
//   piece to the last instead of one burst per wave.
// * kStreamConsumers warps reduce every piece from shared memory: each keeps the masked,
//   NaN-propagating maximum of its share of the piece (packed bf16x2 / f16x2 max, as in
//   WarpSegment) and, only when a piece raises that warp's running maximum, searches the
//   piece for the first element holding it. Pieces of a row arrive in column order, so an
//   equal maximum in a later piece never displaces an earlier index. The consumers then
//   release the stage to the producer ("empty" mbarrier).
// * At the end of a row's part, each consumer warp posts its (maximum, lowest index) pair as
//   one packed key (order << 32 | ~index) in a small ring of row-end slots, and one emitter
//   thread merges them, so the consumers never wait on a global round trip. A row inside
//   one CTA's range is final there; a row split over CTAs is merged through a 16-byte slot
//   in the caller's workspace {key, contributors so far} with a 128-bit compare-and-swap:
//   the CTA whose swap completes the count holds the row's key and writes the outputs, and
//   resets the slot to zero. Verify joins the rows of one batch entry the same way: a
//   16-byte slot per entry holds the miss bits, the count, and the deciding row's
//   selection, so the entry's last row decides from its own swap result. No thread waits
//   on another CTA.
// * Every wait (a stage filling, a stage being released) is bounded by %globaltimer; a CTA
//   that gives up stops waiting altogether, marks its rows ONYX_STATUS_WAIT_TIMEOUT, and its
//   producer waits (bounded) for the copies it issued before the CTA exits.

constexpr int kStreamStages = 6;
constexpr int kStreamConsumers = 16;
constexpr int kStreamProducerWarp = kStreamConsumers;
constexpr int kStreamEmitterWarp = kStreamConsumers + 1;
constexpr int kStreamThreads = (kStreamConsumers + 2) * 32;
constexpr int kStreamRowSlots = 4;  // row ends in flight between the consumers and the emitter
constexpr int kStreamStageBytes = 32768;  // logits bytes per stage
constexpr int kStreamUnit = 256;          // elements per unit
constexpr int kStreamMaskStageBytes = kStreamStageBytes / 2 / 32 * 4 + 16;  // 16-bit pieces
constexpr unsigned long long kStreamWaitLimitNs = 500ull * 1000ull * 1000ull;  // 0.5 s

struct StreamSmem {
  unsigned char x[kStreamStages][kStreamStageBytes];
  unsigned char m[kStreamStages][kStreamMaskStageBytes];
  unsigned long long full[kStreamStages];
  unsigned long long empty[kStreamStages];
  unsigned long long keys[kStreamRowSlots][kStreamConsumers];  // per row end: warp keys
  unsigned long long keys_full[kStreamRowSlots];   // the consumer warps' keys are in
  unsigned long long keys_empty[kStreamRowSlots];  // the emitter has read them
  uint32_t abort;                                  // a wait gave up: stop waiting
};

// ---- mbarrier / bulk-copy helpers (CTA scope) -----------------------------------------
__device__ __forceinline__ void mbar_arrive_cta(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Suspend-time hint of a try_wait: a waiting warp is parked by the hardware until the phase
// completes or this many nanoseconds pass, so waiting costs no issue slots (a plain
// try_wait returns after a short system limit and turns the wait into a polling loop).
constexpr uint32_t kStreamSuspendNs = 1000000u;  // 1 ms

__device__ __forceinline__ bool mbar_try_wait_cta(unsigned long long* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kStreamSuspendNs)
      : "memory");
  return done != 0u;
}

// Waits for phase `parity` of `bar`, bounded; false if it gave up (or another warp of the
// CTA already had: `abort` set), and then sets `abort` so later waits return at once.
__device__ __noinline__ bool stream_wait_slow(unsigned long long* bar, uint32_t parity,
                                              volatile uint32_t* abort) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait_cta(bar, parity)) {
    if (*abort) return false;
    if (global_ns() - t0 > kStreamWaitLimitNs) {
      *abort = 1u;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool stream_wait(unsigned long long* bar, uint32_t parity,
                                            volatile uint32_t* abort) {
  return mbar_try_wait_cta(bar, parity) || stream_wait_slow(bar, parity, abort);
}

// Waits for phase `parity` of `bar` (copies this thread issued), bounded, ignoring `abort`.
__device__ __forceinline__ void stream_drain(unsigned long long* bar, uint32_t parity) {
  if (mbar_try_wait_cta(bar, parity)) return;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait_cta(bar, parity))
    if (global_ns() - t0 > kStreamWaitLimitNs) return;
}

__device__ __forceinline__ unsigned long long l2_evict_first_policy() {
  unsigned long long pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned, size a multiple of 16),
// completion counted on `bar`
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         unsigned long long* bar, unsigned long long policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes,
                                               unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 128-bit compare-and-swap at gpu scope: returns the slot's previous contents
__device__ __forceinline__ ulonglong2 cas128(ulonglong2* addr, ulonglong2 expect,
                                             ulonglong2 desired) {
  ulonglong2 old;
  asm volatile(
      "{\n\t.reg .b128 c, s, d;\n\t"
      "mov.b128 c, {%2, %3};\n\t"
      "mov.b128 s, {%4, %5};\n\t"
      "atom.relaxed.gpu.global.cas.b128 d, [%6], c, s;\n\t"
      "mov.b128 {%0, %1}, d;\n\t}"
      : "=l"(old.x), "=l"(old.y)
      : "l"(expect.x), "l"(expect.y), "l"(desired.x), "l"(desired.y), "l"(addr)
      : "memory");
  return old;
}

// ---- work partition -------------------------------------------------------------------
struct StreamPiece {
  int64_t row;
  int64_t c0, c1;  // columns [c0, c1) of the row
  int64_t next;    // first unit after the piece
  bool row_end;    // last piece of the row inside this CTA's range
};

__device__ __forceinline__ int64_t stream_units_per_row(const ScanParams& p) {
  return (p.vocab + kStreamUnit - 1) / kStreamUnit;
}

// The piece starting at unit u of a range ending at u1.
template <int ES>
__device__ __forceinline__ StreamPiece stream_piece(const ScanParams& p, int64_t upr, int64_t u,
                                                    int64_t u1) {
  constexpr int64_t kUnitsPerPiece = kStreamStageBytes / ES / kStreamUnit;
  StreamPiece q;
  q.row = u / upr;
  const int64_t ru = u - q.row * upr;
  const int64_t row_stop = min(u1, (q.row + 1) * upr);
  const int64_t n = min(row_stop - u, kUnitsPerPiece);
  q.c0 = ru * kStreamUnit;
  q.c1 = min((ru + n) * kStreamUnit, p.vocab);
  q.next = u + n;
  q.row_end = (q.next == row_stop);
  return q;
}

// CTA owning unit u when T units are split over n CTAs as [c T / n, (c + 1) T / n)
__device__ __forceinline__ int64_t stream_owner(int64_t u, int64_t T, int64_t n) {
  return ((u + 1) * n - 1) / T;
}

// Row r's logits
template <int MODE, int ES>
__device__ __forceinline__ const char* stream_row_logits(const ScanParams& p, int64_t r) {
  if constexpr (MODE == kModeVerify) {
    const int64_t g = r / p.per_group, i = r - g * p.per_group;
    return static_cast<const char*>(p.logits) + (g * p.group_stride + i * p.row_stride) * ES;
  }
  return static_cast<const char*>(p.logits) + r * p.group_stride * ES;
}

// Row r's mask words. A gather row whose DFA state id lies outside the table reads table
// row 0 instead (the consumers skip the row and its outputs report BAD_STATE).
template <int MODE>
__device__ __forceinline__ const uint32_t* stream_row_mask(const ScanParams& p, int64_t r) {
  if constexpr (MODE == kModeVerify) {
    const int64_t g = r / p.per_group, i = r - g * p.per_group;
    return p.mask + g * p.mask_group_stride + i * p.mask_row_stride;
  }
  if (p.state_ids) {
    const int32_t s = __ldg(p.state_ids + r);
    const bool bad = (s < 0) || ((int64_t)s >= p.n_states);
    return p.mask + (bad ? 0 : (int64_t)s * p.mask_row_stride);
  }
  return p.mask + r * p.mask_group_stride;
}

// Bytes of a piece's logits and mask-word copies
template <int ES>
__device__ __forceinline__ void stream_piece_bytes(const StreamPiece& q, uint32_t* xb,
                                                   uint32_t* mb) {
  *xb = (uint32_t)((q.c1 - q.c0) * ES);
  const int64_t w0 = q.c0 >> 5, w1 = (q.c1 + 31) >> 5;
  *mb = (uint32_t)(((w1 - w0) * 4 + 15) & ~15ll);
}

// ---- outputs --------------------------------------------------------------------------
__device__ __forceinline__ Partial key_to_partial(unsigned long long key) {
  Partial pr;
  pr.flags = (key == kKeyWaitTimeout ? kFlagWaitTimeout : 0u) | (key ? kFlagAny : 0u);
  pr.ord = key >> 32;
  pr.idx = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
  return pr;
}

// The row's final key is known: write the row's outputs (argmax / key modes) or join the
// row's batch entry (verify). One thread.
template <int MODE>
__device__ void stream_emit_final(const ScanParams& p, int64_t r, unsigned long long key) {
  if constexpr (MODE == kModeArgmax) {
    Partial pr = key_to_partial(key);
    if (p.state_ids) {
      const int32_t s = __ldg(p.state_ids + r);
      if ((s < 0) || ((int64_t)s >= p.n_states)) pr.flags |= kFlagBadState;
    }
    decode_partial(pr, false, &p.out_idx[r], &p.out_status[r]);
  } else if constexpr (MODE == kModeKey) {
    if (p.n_key_dst) {
      if (__ldcg(p.key_failed) == 0ull) {  // a failed exchange stores no key anywhere
        const int64_t slot = ((__ldcg(p.key_epoch) + 1ull) & 1ull ? p.key_parity_stride : 0) + r;
        for (int i = 0; i < p.n_key_dst; ++i) p.key_dst[i][slot] = key;
      }
    } else {
      p.out_key[r] = key;
    }
  } else {
    // verify: this row's decision inputs, merged into its entry's slot
    const int P = p.per_group, G = P - 1;
    const int64_t g = r / P;
    const int i = (int)(r - g * P);
    int32_t sel;
    uint32_t rs;
    decode_partial(key_to_partial(key), false, &sel, &rs);
    const bool miss = i < G && (rs != 0u || sel != __ldg(p.drafts + g * p.draft_stride + i));
    const bool cand = miss || i == G;  // the deciding row is the lowest of these
    // slot.x: miss bits [0, 32) | count [32, 40) | candidate row [40, 48) | its status
    //         [48, 56) | has candidate (bit 56); slot.y: the candidate's selection
    ulonglong2* slot = p.group_slots + g;
    ulonglong2 cur = make_ulonglong2(0ull, 0ull);
    ulonglong2 nxt;
    for (;;) {
      nxt = cur;
      if (miss) nxt.x |= 1ull << i;
      nxt.x += 1ull << 32;
      const bool has = (cur.x >> 56) & 1ull;
      const int crow = (int)((cur.x >> 40) & 0xFFull);
      if (cand && (!has || i < crow)) {
        nxt.x = (nxt.x & 0x000000FFFFFFFFFFull) | ((unsigned long long)i << 40) |
                ((unsigned long long)(rs & 0xFFu) << 48) | (1ull << 56);
        nxt.y = (unsigned long long)(uint32_t)sel;
      }
      const ulonglong2 old = cas128(slot, cur, nxt);
      if (old.x == cur.x && old.y == cur.y) break;
      cur = old;
    }
    if ((int)((nxt.x >> 32) & 0xFFull) != P) return;
    // the entry's last row: decide and reset the slot
    const uint32_t miss_bits = (uint32_t)(nxt.x & 0xFFFFFFFFull) & ((G >= 32) ? 0xFFFFFFFFu : ((1u << G) - 1u));
    const int acc = miss_bits ? __ffs(miss_bits) - 1 : G;
    int32_t corr = -1;
    uint32_t st = 0u;
    if (acc < G || p.bonus) {
      const uint32_t crs = (uint32_t)((nxt.x >> 48) & 0xFFull);
      if (crs) {
        st = crs;
      } else {
        corr = (int32_t)(uint32_t)nxt.y;
      }
    }
    p.accept_len[g] = acc;
    p.correction[g] = corr;
    p.out_status[g] = st;
    __stcg(slot, make_ulonglong2(0ull, 0ull));
  }
}

// A row part's key from this CTA: final if the CTA covers the whole row, else merged into
// the row's workspace slot. One thread.
template <int MODE>
__device__ void stream_emit_part(const ScanParams& p, int64_t r, unsigned long long key,
                                 int64_t upr, int64_t T, int64_t n) {
  const int64_t first = stream_owner(r * upr, T, n);
  const int64_t last = stream_owner((r + 1) * upr - 1, T, n);
  const unsigned long long parts = (unsigned long long)(last - first + 1);
  if (parts == 1ull) {
    stream_emit_final<MODE>(p, r, key);
    return;
  }
  ulonglong2* slot = p.row_slots + r;
  ulonglong2 cur = make_ulonglong2(0ull, 0ull);
  ulonglong2 nxt;
  for (;;) {
    nxt = make_ulonglong2(cur.x > key ? cur.x : key, cur.y + 1ull);
    const ulonglong2 old = cas128(slot, cur, nxt);
    if (old.x == cur.x && old.y == cur.y) break;
    cur = old;
  }
  if (nxt.y != parts) return;
  __stcg(slot, make_ulonglong2(0ull, 0ull));  // every contributor has merged: reset
  stream_emit_final<MODE>(p, r, nxt.x);
}

// ---- the kernel ---------------------------------------------------------------------------
template <int DT, int MODE>
__global__ void __launch_bounds__(kStreamThreads, 1) masked_stream_kernel(const ScanParams p) {
  static_assert(DT == kBF16 || DT == kF16 || DT == kF32, "16-byte vector types only");
  constexpr int ES = (DT == kF32) ? 4 : 2;
  using V = Vec16<DT>;
  constexpr int E = V::kElems;                                  // elements per 16-byte vector
  constexpr int kVecPerPiece = kStreamStageBytes / 16;          // 2048
  constexpr int kVecPerLane = kVecPerPiece / (kStreamConsumers * 32);  // 4
  constexpr uint32_t kLaneBits = (E == 8) ? 0xFFu : 0xFu;
  extern __shared__ __align__(128) unsigned char stream_smem_raw[];
  StreamSmem& S = *reinterpret_cast<StreamSmem*>(stream_smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStreamStages; ++s) {
      mbar_init(&S.full[s], 1u);
      mbar_init(&S.empty[s], (uint32_t)kStreamConsumers);
    }
    for (int s = 0; s < kStreamRowSlots; ++s) {
      mbar_init(&S.keys_full[s], (uint32_t)kStreamConsumers);
      mbar_init(&S.keys_empty[s], 1u);
    }
    S.abort = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Programmatic dependent launch: everything read below may come from the preceding kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" :::);

  const int64_t T = p.rows * stream_units_per_row(p);
  const int64_t n = gridDim.x;
  const int64_t upr = stream_units_per_row(p);
  const int64_t u0 = (int64_t)blockIdx.x * T / n, u1 = ((int64_t)blockIdx.x + 1) * T / n;
  volatile uint32_t* abort = &S.abort;

  if (warp == kStreamEmitterWarp) {
    // ---------------- emitter: one thread ----------------
    // Row ends in the consumers' order: merge the warps' keys, then write the row's outputs
    // or merge it into its workspace slot. The compare-and-swap round trips happen here, so
    // the consumers never wait for them.
    if (lane != 0) return;
    int64_t re = 0;
    for (int64_t u = u0; u < u1;) {
      const StreamPiece q = stream_piece<ES>(p, upr, u, u1);
      u = q.next;
      if (!q.row_end) continue;
      const int i = (int)(re % kStreamRowSlots);
      const uint32_t par = (uint32_t)((re / kStreamRowSlots) & 1);
      unsigned long long key;
      if (stream_wait(&S.keys_full[i], par, abort)) {
        key = 0ull;
#pragma unroll
        for (int w = 0; w < kStreamConsumers; ++w) key = S.keys[i][w] > key ? S.keys[i][w] : key;
      } else {
        key = kKeyWaitTimeout;
      }
      mbar_arrive_cta(&S.keys_empty[i]);
      stream_emit_part<MODE>(p, q.row, key, upr, T, n);
      ++re;
    }
    return;
  }

  if (warp == kStreamProducerWarp) {
    // ---------------- producer: one thread ----------------
    if (lane != 0) return;
    const unsigned long long pol = l2_evict_first_policy();
    // the logits copies of the first stages go out before anything that needs a dependent
    // load (a gather row's DFA state id)
    {
      int64_t u = u0;
      for (int j = 0; j < kStreamStages && u < u1; ++j) {
        const StreamPiece q = stream_piece<ES>(p, upr, u, u1);
        u = q.next;
        uint32_t xb, mb;
        stream_piece_bytes<ES>(q, &xb, &mb);
        mbar_arrive_expect_tx(&S.full[j], xb + mb);
        bulk_g2s(S.x[j], stream_row_logits<MODE, ES>(p, q.row) + q.c0 * ES, xb, &S.full[j], pol);
      }
    }
    int64_t k = 0;
    int64_t cur_row = -1;
    const uint32_t* mrow = nullptr;
    for (int64_t u = u0; u < u1; ++k) {
      const StreamPiece q = stream_piece<ES>(p, upr, u, u1);
      u = q.next;
      const int s = (int)(k % kStreamStages);
      uint32_t xb, mb;
      stream_piece_bytes<ES>(q, &xb, &mb);
      if (k >= kStreamStages) {
        if (*abort || !stream_wait(&S.empty[s], (uint32_t)((k / kStreamStages - 1) & 1), abort))
          break;  // the consumers gave up: issue nothing more
        mbar_arrive_expect_tx(&S.full[s], xb + mb);
        bulk_g2s(S.x[s], stream_row_logits<MODE, ES>(p, q.row) + q.c0 * ES, xb, &S.full[s], pol);
      }
      if (q.row != cur_row) {
        cur_row = q.row;
        mrow = stream_row_mask<MODE>(p, q.row);
      }
      bulk_g2s_plain(S.m[s], mrow + (q.c0 >> 5), mb, &S.full[s]);
    }
    // the copies issued into the last stages have landed before this CTA may exit
    const int64_t issued = k;
    for (int64_t j = issued - 1; j >= 0 && j >= issued - kStreamStages; --j)
      stream_drain(&S.full[j % kStreamStages], (uint32_t)((j / kStreamStages) & 1));
    return;
  }

  // ---------------- consumers ----------------
  uint32_t best_ord = 0u, best_idx = 0xFFFFFFFFu;
  bool gave_up = false;
  int row_ends = 0;
  int64_t k = 0;
  for (int64_t u = u0; u < u1; ++k) {
    const StreamPiece q = stream_piece<ES>(p, upr, u, u1);
    u = q.next;
    const int s = (int)(k % kStreamStages);
    const bool ok = !gave_up && stream_wait(&S.full[s], (uint32_t)((k / kStreamStages) & 1), abort);
    gave_up = !ok;
    bool bad = false;
    if (ok && MODE == kModeArgmax && p.state_ids) {
      const int32_t sid = __ldg(p.state_ids + q.row);
      bad = (sid < 0) || ((int64_t)sid >= p.n_states);
    }
    if (ok && !bad) {
      const int nvec = (int)((q.c1 - q.c0) / E);
      const uint4* xs = reinterpret_cast<const uint4*>(S.x[s]);
      const uint32_t* ms = reinterpret_cast<const uint32_t*>(S.m[s]);
      uint4 x[kVecPerLane];
      uint32_t bits[kVecPerLane];
      uint32_t vm[kVecPerLane];
      float tmax = __int_as_float(0xFF800000);
      uint32_t pm = 0u;
      if constexpr (DT != kF32) pm = V::kNegInfPair;
      uint32_t any = 0u;
#pragma unroll
      for (int j = 0; j < kVecPerLane; ++j) {
        const int v = (j * kStreamConsumers + warp) * 32 + lane;
        if (v < nvec) {
          x[j] = xs[v];
          bits[j] = (ms[(v * E) >> 5] >> ((v * E) & 31)) & kLaneBits;
        } else {
          x[j] = make_uint4(0u, 0u, 0u, 0u);
          bits[j] = 0u;
        }
        any |= bits[j];
        if constexpr (DT == kF32) {
          tmax = max_nan_f32(tmax, V::masked_max(x[j], bits[j]));
        } else {
          vm[j] = V::masked_pair_max(x[j], bits[j]);
          pm = V::pmax(pm, vm[j]);
        }
      }
      if constexpr (DT != kF32) tmax = V::pair_to_f32_max(pm);
      const uint32_t tord = any ? ord32(tmax) : 0u;
      const uint32_t M = __reduce_max_sync(kFull, tord);
      if (M > best_ord) {
        uint32_t idx = 0xFFFFFFFFu;
        if (M != kOrd32NaN) {
          // first (vector j, lane) whose masked maximum is M, then its first valid element
          const float mf = __uint_as_float((M & 0x80000000u) ? (M & 0x7FFFFFFFu) : ~M);
          uint32_t keyjl = 0xFFFFFFFFu;
          if (tord == M) {
#pragma unroll
            for (int j = kVecPerLane - 1; j >= 0; --j) {
              bool hit;
              if constexpr (DT == kF32) {
                hit = bits[j] && V::masked_max(x[j], bits[j]) == mf;
              } else {
                const uint32_t h = V::from_f32(mf);
                hit = bits[j] && V::eq_mask(vm[j], h | (h << 16));
              }
              if (hit) keyjl = ((uint32_t)j << 5) | (uint32_t)lane;
            }
          }
          const uint32_t win = __reduce_min_sync(kFull, keyjl);
          const int wj = (int)(win >> 5), wl = (int)(win & 31u);
          uint4 xv = x[0];
          uint32_t bv = bits[0];
#pragma unroll
          for (int j = 1; j < kVecPerLane; ++j)
            if (j == wj) {
              xv = x[j];
              bv = bits[j];
            }
          int e;
          if constexpr (DT == kF32) {
            e = 3;
            if ((bv & 4u) && __uint_as_float(xv.z) == mf) e = 2;
            if ((bv & 2u) && __uint_as_float(xv.y) == mf) e = 1;
            if ((bv & 1u) && __uint_as_float(xv.x) == mf) e = 0;
          } else {
            const uint32_t h = V::from_f32(mf);
            const uint32_t m2 = h | (h << 16);
            uint32_t m01, m23, m45, m67;
            expand8_16(bv, m01, m23, m45, m67);
            const uint32_t q0 = V::eq_mask(xv.x, m2) & m01;
            const uint32_t q1 = V::eq_mask(xv.y, m2) & m23;
            const uint32_t q2 = V::eq_mask(xv.z, m2) & m45;
            const uint32_t q3 = V::eq_mask(xv.w, m2) & m67;
            const unsigned long long lo = (unsigned long long)q0 | ((unsigned long long)q1 << 32);
            const unsigned long long hi = (unsigned long long)q2 | ((unsigned long long)q3 << 32);
            e = lo ? (__ffsll((long long)lo) - 1) >> 4 : 4 + ((__ffsll((long long)hi) - 1) >> 4);
          }
          e = __shfl_sync(kFull, e, wl);
          const int v = (wj * kStreamConsumers + warp) * 32 + wl;
          idx = (uint32_t)(q.c0 + (int64_t)v * E + e);
        }
        best_ord = M;
        best_idx = idx;
      }
    }
    // this warp is done with the stage
    __syncwarp();
    if (lane == 0) mbar_arrive_cta(&S.empty[s]);

    if (q.row_end) {
      // merge the consumer warps' (maximum, lowest index) of this row part
      unsigned long long wkey = 0ull;
      if (best_ord) {
        const uint32_t gidx = best_idx == 0xFFFFFFFFu ? best_idx : best_idx + (uint32_t)p.idx_offset;
        wkey = ((unsigned long long)best_ord << 32) | (0xFFFFFFFFull - gidx);
      }
      if (gave_up) wkey = kKeyWaitTimeout;
      // hand the key to the emitter through the row-end ring
      const int i = row_ends % kStreamRowSlots;
      if (lane == 0) {
        if (row_ends >= kStreamRowSlots &&
            !stream_wait(&S.keys_empty[i], (uint32_t)((row_ends / kStreamRowSlots - 1) & 1), abort))
          wkey = kKeyWaitTimeout;  // the slot is stale: the emitter's wait gives up too
        S.keys[i][warp] = wkey;
        mbar_arrive_cta(&S.keys_full[i]);
      }
      __syncwarp();
      ++row_ends;
      best_ord = 0u;
      best_idx = 0xFFFFFFFFu;
    }
  }
}
