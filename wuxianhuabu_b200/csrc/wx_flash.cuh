// wx_flash.cuh — shared pieces of the tcgen05 flash-attention kernels (included
// by wx_attn.cu before wx_flash2.cuh and wx_flash5.cuh): the launch parameters,
// the key-tile walk of a work item, the output-row destination (local or another
// rank's memory), the MUFU exponential and the register split of the 12-warp
// kernels.
#pragma once

constexpr int kAttnThreads = 192;          // flash_attn2_kernel: TMA, MMA, 4 softmax warps
constexpr int kTileBytes = 128 * 128 * 2;  // one 128x128 bf16 operand tile (head_dim 128)
constexpr int kChunkBytes = 128 * 128;     // one 64-column SW128 chunk of a 128-row tile
constexpr int kHalfBytes = 64 * 128;       // 64 rows of such a chunk (one TMA box)

struct AttnParams {
  const WorkItem* items;
  const int4* entries;
  const float* tailT;
  const float* tailL;
  const float* tailC;
  int nqb;
  int H;
  float sl2;  // softmax scale * log2(e)
  __nv_bfloat16* out;
  int64_t out_stride;
  int* err;
  // Sequence parallelism over peer memory (paired / duo kernels): query row s is
  // written to rank s / peer_rows at out_peer[r] + (s - r*peer_rows)*out_stride +
  // peer_col + head*head_dim; out_peer[0] == nullptr writes to `out`. sig.counter !=
  // nullptr: the last CTA of the call signals every rank (peer_signal_cta_done).
  __nv_bfloat16* out_peer[kMaxPeers];
  int64_t peer_rows;
  int peer_col;
  PeerSignal sig;
  // extents the bounds-checked build tests against: query rows of the sequence, list
  // entries, ranks receiving rows (0 = local output)
  int64_t S;
  int64_t n_entries;
  int P;
};

// (bounds-checked build) output row `row` has a destination
__device__ __forceinline__ bool attn_row_ok(const AttnParams& p, int64_t row) {
  if (row < 0 || row >= p.S) return false;
  if (p.out_peer[0] == nullptr) return true;
  const int64_t owner = row / p.peer_rows;
  return owner < p.P && owner < kMaxPeers && p.out_peer[owner] != nullptr;
}

// destination of output row `row` (query row of the sequence) of head `head`
template <int HD>
__device__ __forceinline__ __nv_bfloat16* attn_out_row(const AttnParams& p, int64_t row, int head) {
  if (p.out_peer[0] == nullptr) return p.out + row * p.out_stride + head * HD;
  const int64_t owner = row / p.peer_rows;
  __nv_bfloat16* base = p.out_peer[0];
#pragma unroll
  for (int r = 1; r < kMaxPeers; ++r)
    if (owner == r) base = p.out_peer[r];
  return base + (row - owner * p.peer_rows) * p.out_stride + p.peer_col + head * HD;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// three-input max (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// key tile j of a work item: two 64-row halves (start row, valid length | q-half mask << 8)
__device__ __forceinline__ int4 kv_entry(const WorkItem& it, const AttnParams& p, int j) {
  if (j < it.n_implicit) {
    const int s0 = j * 128;
    return make_int4(s0, s0 + 64, max(0, min(64, it.implicit_end - s0)) | (3 << 8),
                     max(0, min(64, it.implicit_end - s0 - 64)) | (3 << 8));
  }
  const int64_t idx = (int64_t)it.list_begin + (j - it.n_implicit);
  if (!WX_IN_BOUNDS(p.err, idx >= 0 && idx < p.n_entries)) return make_int4(0, 0, 0, 0);  // (empty halves)
  return __ldg(p.entries + idx);
}

__device__ __forceinline__ int item_tiles(const WorkItem& it) { return it.n_implicit + it.list_len; }

// a value the compiler must recompute where it is used (keeps MMA descriptors
// out of registers between uses instead of hoisting all of them)
__device__ __forceinline__ uint64_t opaque64(uint64_t v) {
  uint64_t r;
  asm volatile("mov.b64 %0, %1;" : "=l"(r) : "l"(v));
  return r;
}

// Register split of the 384-thread kernels: warps 0-3 (TMA, MMA issuers) give
// registers up, the eight softmax warps take them (72*128 + 216*256 = 168*384).
constexpr int kA5Threads = 384;
constexpr int kRegsLow = 72;
constexpr int kRegsHigh = 216;
static_assert(kRegsLow * 128 + kRegsHigh * 256 <= 168 * kA5Threads, "register split exceeds the launch");

__device__ __forceinline__ void reg_dealloc_low() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
}
__device__ __forceinline__ void reg_alloc_high() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
}
