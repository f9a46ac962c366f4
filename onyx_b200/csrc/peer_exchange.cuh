// Vocabulary-sharded selection with the key exchange done over NVLink peer memory
// (included by masked_select.cu inside namespace onyx, after the combine kernel).
//
// Every rank owns one exchange buffer, allocated with cudaMalloc and mapped into every
// other rank's address space through CUDA IPC:
//
//   [flags: kMaxExchangeRanks x u64 | epoch count: u64 at byte 128 | failed: u64 at byte
//    136 | ... 256 bytes]
//   [slots: 2 parities x world x rows_cap x u64]
//
// The epoch count is this rank's number of finished calls; call e is the count + 1, read on
// the device, so a captured CUDA graph replays correctly. One call (epoch e, the same on
// every rank since all make the same calls, parity e & 1):
//   1. the shard-key kernel (key mode) stores row r's key into slot [parity][rank][r] of every
//      rank's buffer -- plain stores, the peers' over NVLink -- instead of a local key array;
//   2. exchange_combine_kernel (one CTA, next in the stream) raises this rank's flag to e in
//      every rank's buffer (one fence.acq_rel.sys, then relaxed system-scope stores, all in
//      flight together), waits until every flag in its own buffer is >= e (lane i of warp 0
//      polls rank i's flag with ld.acquire.sys, bounded; a block barrier then orders the
//      whole block after those acquires), combines the world keys of each row from its own
//      buffer into the outputs, and stores e as the new epoch count.
// A rank reaches call e + 1's stores only after seeing every rank's flag for e, which every
// rank raises after its own call e - 1 finished reading; with two parities no store can
// land in a slot a peer is still reading. Flags only grow, so a rank that has moved on
// to e + 1 never hides e from a slower peer.
//
// A wait that gives up breaks that invariant (this rank no longer knows which slots its
// peers read), so the failure is sticky: the exchange kernel sets this rank's "failed"
// word and leaves the epoch count where it was; from then on the shard kernel stores no
// key into any buffer and the exchange kernel neither raises flags nor waits -- every row
// of every later call reports ONYX_STATUS_WAIT_TIMEOUT until the ranks build new buffers.
// Peers waiting on this rank's flag give up in turn and fail the same way.

constexpr int kMaxExchangeRanks = 8;
constexpr size_t kExchangeFlagBytes = 256;
constexpr size_t kExchangeEpochOffset = 128;  // this rank's count of finished calls
constexpr size_t kExchangeFailedOffset = 136;  // nonzero once a wait of this rank gave up
constexpr unsigned long long kExchangeWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

struct ExchangeParams {
  unsigned long long* own_flags;               // this rank's buffer: one flag per rank
  unsigned long long* own_epoch;               // this rank's buffer: finished calls
  unsigned long long* own_failed;              // this rank's buffer: sticky failure
  unsigned long long* flag_dst[kMaxExchangeRanks];  // this rank's flag in every rank's buffer
  const unsigned long long* slots;             // this rank's buffer, parity 0
  int64_t parity_stride;                       // world * rows_cap
  int world;
  int64_t rows;
  int64_t rows_cap;
  int32_t* out_idx;
  uint32_t* out_status;
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(1024) exchange_combine_kernel(const ExchangeParams e) {
  __shared__ uint32_t s_ok;
  __shared__ unsigned long long s_epoch;
  // the shard-key kernel, and with it this rank's stores into every buffer, has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const unsigned long long epoch = __ldcg(e.own_epoch) + 1ull;
    bool ok = __ldcg(e.own_failed) == 0ull;  // (the same word for every lane)
    if (ok) {
      // release: one system fence, then this rank's flag in every buffer (relaxed stores
      // after the fence, all in flight at once)
      if (lane == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int i = 0; i < e.world; ++i) st_relaxed_sys_u64(e.flag_dst[i], epoch);
      }
      // acquire: lane i waits for rank i's flag in this rank's buffer, all ranks at once
      bool arrived = true;
      if (lane < e.world) {
        const unsigned long long t0 = global_ns();
        while (ld_acquire_sys_u64(e.own_flags + lane) < epoch) {
          if (global_ns() - t0 > kExchangeWaitLimitNs) {
            arrived = false;
            break;
          }
        }
      }
      ok = __all_sync(0xFFFFFFFFu, arrived);
      if (!ok && lane == 0) __stcg(e.own_failed, 1ull);  // sticky: later calls neither store nor wait
    }
    if (lane == 0) {
      s_epoch = epoch;
      s_ok = ok ? 1u : 0u;
    }
  }
  __syncthreads();  // (extends each lane's acquire to the whole block)
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const bool ok = s_ok != 0u;
  const unsigned long long* slots = e.slots + ((s_epoch & 1ull) ? e.parity_stride : 0);
  for (int64_t r = threadIdx.x; r < e.rows; r += blockDim.x) {
    unsigned long long k[kMaxExchangeRanks];
#pragma unroll
    for (int i = 0; i < kMaxExchangeRanks; ++i)
      k[i] = i < e.world ? __ldcg(slots + (int64_t)i * e.rows_cap + r) : 0ull;
    unsigned long long best = 0ull;
#pragma unroll
    for (int i = 0; i < kMaxExchangeRanks; ++i) best = k[i] > best ? k[i] : best;
    Partial pr;
    pr.flags = (best == kKeyWaitTimeout || !ok ? kFlagWaitTimeout : 0u) | (best ? kFlagAny : 0u);
    pr.ord = best >> 32;
    pr.idx = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    decode_partial(pr, false, &e.out_idx[r], &e.out_status[r]);
  }
  // the next call's shard kernel reads the count for its parity; a failed exchange keeps it
  if (threadIdx.x == 0 && ok) __stcg(e.own_epoch, s_epoch);
}
