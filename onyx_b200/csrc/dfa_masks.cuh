// Valid-token bitmasks of DFA states on the GPU (included by masked_select.cu inside
// namespace onyx). Restates the reference's valid-id scan,
// onyx_cuda/rust/src/regex_runtime.rs:129-145 with the transition fold of :197-201: a
// token is valid from state s iff it is non-empty and walking its bytes through the dense
// transition table from s does not end in the dead state. Row r of the output is the
// packed mask (bit t of word t >> 5, LSB first, tail bits zero) of states[r].
//
// One warp builds one 32-token mask word for up to kDfaMaxRowsPerWarp states: each lane loads
// its token once and walks it from kDfaLockstep states at a time in lockstep, so their table
// loads (read-only path; a regex DFA of a few hundred states stays in L1) overlap, and a
// ballot packs each row's word. When the dead state is absorbing a walk stops at it; otherwise the full token is
// walked, which is the reference's final-state rule in both cases. A transition outside
// the table counts as the dead state and a token whose offsets leave the byte array counts
// as empty, so malformed input cannot send a load out of bounds; a state id outside the
// table yields an empty row.

constexpr int kDfaMaxRowsPerWarp = 32;  // state rows one warp builds for its token word
constexpr int kDfaLockstep = 4;         // of which walked together
constexpr int kDfaWarpsPerBlock = 8;
constexpr int kDfaCachedBytes = 16;  // token bytes kept in registers; longer tails re-read

struct DfaParams {
  const int32_t* trans;  // [n_states][256] next state
  int32_t n_states;
  int32_t dead;
  int dead_absorbing;  // every transition from dead returns to dead
  const int32_t* states;  // [rows]
  int64_t rows;
  const uint8_t* tok_bytes;
  int64_t n_bytes;             // size of tok_bytes
  const int64_t* tok_offsets;  // [vocab + 1]
  int64_t vocab;
  uint32_t* out;  // [rows][out_stride] words
  int64_t out_stride;
  int rows_per_warp;  // a multiple of kDfaLockstep, at most kDfaMaxRowsPerWarp
};

__global__ void __launch_bounds__(kDfaWarpsPerBlock * 32) dfa_mask_kernel(const DfaParams d) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t word = (int64_t)blockIdx.x * kDfaWarpsPerBlock + (threadIdx.x >> 5);
  const int64_t words = (d.vocab + 31) / 32;
  if (word >= words) return;  // warp-uniform
  const int64_t row0 = (int64_t)blockIdx.y * d.rows_per_warp;
  const int64_t t = word * 32 + lane;

  // this lane's token: length and its first bytes in registers
  int64_t a = 0, len = 0;
  if (t < d.vocab) {
    a = __ldg(d.tok_offsets + t);
    len = __ldg(d.tok_offsets + t + 1) - a;
    if (a < 0 || len < 0 || a + len > d.n_bytes) len = 0;  // malformed offsets: no token
  }
  uint32_t cached[kDfaCachedBytes / 4];
#pragma unroll
  for (int i = 0; i < kDfaCachedBytes / 4; ++i) cached[i] = 0u;
#pragma unroll
  for (int i = 0; i < kDfaCachedBytes; ++i)
    if (i < len) cached[i >> 2] |= (uint32_t)__ldg(d.tok_bytes + a + i) << (8 * (i & 3));

  // the walks, kDfaLockstep state rows at a time, the token bytes reused for all of them
  const int64_t row_end = min(d.rows, row0 + (int64_t)d.rows_per_warp);
  for (int64_t rg = row0; rg < row_end; rg += kDfaLockstep) {
    int32_t s[kDfaLockstep];
    bool live[kDfaLockstep];
#pragma unroll
    for (int j = 0; j < kDfaLockstep; ++j) {
      const int64_t r = rg + j;
      const int32_t st = r < row_end ? __ldg(d.states + r) : -1;
      const bool ok = st >= 0 && st < d.n_states;
      s[j] = ok ? st : d.dead;
      live[j] = ok && len > 0 && !(d.dead_absorbing && st == d.dead);
    }
    // one byte of every live walk: 32-bit table offsets (the host bounds n_states * 256
    // below 2^31); an entry outside the table is the dead state
    auto step = [&](uint32_t b) {
#pragma unroll
      for (int j = 0; j < kDfaLockstep; ++j) {
        if (!live[j]) continue;
        int32_t nx = __ldg(d.trans + (((uint32_t)s[j] << 8) | b));
        if ((uint32_t)nx >= (uint32_t)d.n_states) nx = d.dead;
        s[j] = nx;
        if (d.dead_absorbing && nx == d.dead) live[j] = false;
      }
    };
    auto any_live = [&]() {
      bool any = false;
#pragma unroll
      for (int j = 0; j < kDfaLockstep; ++j) any |= live[j];
      return any;
    };
    // the cached bytes four at a time (fixed shifts), then any longer tail from memory
    const int lc = (int)min(len, (int64_t)kDfaCachedBytes);
#pragma unroll
    for (int q = 0; q < kDfaCachedBytes / 4; ++q) {
      if (q * 4 >= lc || !any_live()) break;
      const uint32_t w = cached[q];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (q * 4 + k < lc) step((w >> (8 * k)) & 0xFFu);
    }
    for (int64_t i = kDfaCachedBytes; i < len && any_live(); ++i) step(__ldg(d.tok_bytes + a + i));
#pragma unroll
    for (int j = 0; j < kDfaLockstep; ++j) {
      const int64_t r = rg + j;
      // rows past the end and state ids outside the table start (and stay) at dead
      const bool valid = t < d.vocab && len > 0 && s[j] != d.dead;
      const uint32_t bits = __ballot_sync(kFull, valid);
      if (lane == 0 && r < row_end) d.out[r * d.out_stride + word] = bits;
    }
  }
}
