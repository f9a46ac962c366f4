// Vocabulary-sharded selection with the key exchange done over NVLink peer memory
// (included by masked_select.cu inside namespace onyx, after the combine kernel).
//
// Every rank owns one exchange buffer, allocated with cudaMalloc and mapped into every
// other rank's address space through CUDA IPC:
//
//   [flags: kMaxExchangeRanks x u64, 256 bytes][slots: 2 parities x world x rows_cap x u64]
//
// One call (epoch e >= 1, the same on every rank, parity e & 1):
//   1. the shard-key kernel (key mode) stores row r's key into slot [parity][rank][r] of every
//      rank's buffer -- plain stores, the peers' over NVLink -- instead of a local key array;
//   2. exchange_combine_kernel (one CTA, next in the stream) raises this rank's flag to e in
//      every rank's buffer (fence.acq_rel.sys, then st.release.sys), waits until every flag
//      in its own buffer is >= e (ld.acquire.sys, bounded), and combines the world keys of
//      each row from its own buffer into the outputs.
// A rank reaches call e + 1's stores only after seeing every rank's flag for e, which every
// rank raises after its own call e - 1 finished reading; with two parities no store can
// land in a slot a peer is still reading. Flags only grow, so a rank that has moved on
// to e + 1 never hides e from a slower peer.

constexpr int kMaxExchangeRanks = 8;
constexpr size_t kExchangeFlagBytes = 256;
constexpr unsigned long long kExchangeWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

struct ExchangeParams {
  unsigned long long* own_flags;               // this rank's buffer: one flag per rank
  unsigned long long* flag_dst[kMaxExchangeRanks];  // this rank's flag in every rank's buffer
  const unsigned long long* slots;             // this rank's buffer, this call's parity
  int world;
  int64_t rows;
  int64_t rows_cap;
  unsigned long long epoch;
  int32_t* out_idx;
  uint32_t* out_status;
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(1024) exchange_combine_kernel(const ExchangeParams e) {
  __shared__ uint32_t s_ok;
  // the shard-key kernel, and with it this rank's stores into every buffer, has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int i = 0; i < e.world; ++i) st_release_sys_u64(e.flag_dst[i], e.epoch);
    bool ok = true;
    const unsigned long long t0 = global_ns();
    for (int i = 0; i < e.world && ok; ++i) {
      while (ld_acquire_sys_u64(e.own_flags + i) < e.epoch) {
        if (global_ns() - t0 > kExchangeWaitLimitNs) {
          ok = false;
          break;
        }
      }
    }
    s_ok = ok ? 1u : 0u;
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const bool ok = s_ok != 0u;
  for (int64_t r = threadIdx.x; r < e.rows; r += blockDim.x) {
    unsigned long long best = 0ull;
    for (int i = 0; i < e.world; ++i) {
      const unsigned long long k = __ldcg(e.slots + (int64_t)i * e.rows_cap + r);
      best = k > best ? k : best;
    }
    Partial pr;
    pr.flags = (best == kKeyWaitTimeout || !ok ? kFlagWaitTimeout : 0u) | (best ? kFlagAny : 0u);
    pr.ord = best >> 32;
    pr.idx = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    decode_partial(pr, false, &e.out_idx[r], &e.out_status[r]);
  }
}
