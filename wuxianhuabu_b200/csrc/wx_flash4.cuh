// wx_flash4.cuh — persistent flash-attention kernel, one CTA per SM, one work
// item at a time, with the softmax of each key tile split over two warpgroups
// by columns (included by wx_attn.cu after wx_flash.cuh, whose helpers it shares).
//
// Per 128-key tile the tensor pipe needs 1024 cycles (S = Q K^T, O += P V) and
// one 4-warp softmax needs ~1500 (one exp2 per score on MUFU plus the TMEM
// round trip), so a softmax that waits for its own PV / next S (P aliasing S)
// leaves the tensor pipe half idle. Here:
//   TMEM (512 columns): S double buffer [0,128) [128,256); P double buffer
//   (packed bf16) [256,320) [320,384); O [384,512).
//   S(t+2) is issued as soon as the softmax has read S(t) into registers, and
//   PV(t) as soon as P(t) is written, so the tensor pipe computes S(t+2) and
//   PV(t) while the softmax works on t+1.
//   Warpgroup w (warps 4w+4 .. 4w+7, w = 0, 1) exponentiates key columns
//   [64w, 64w+64) of every tile: both read the whole row of S for the row max
//   (no exchange needed), each writes its half of P, keeps its half of the row
//   sum, rescales its half of O (lazy, when the max grew by more than 2^8) and
//   stores its half of the output row.
//   Warp 0: TMA producer (Q, K ring of 3, V ring of 3, L2 prefetch ahead) and the
//   dynamic work-item fetch (atomic counter, 2-deep queue in shared memory).
//   Warp 1: issues S = Q K^T (and owns TMEM); warp 2: issues O += P V; warp 3 idle.
// S(t) needs K(t) and S buffer t&1 (read by the softmax of t-2); PV(t) needs
// P(t) and V(t). The producer loads K(0), K(1), then K(t+2), V(t) per tile t;
// every load waits only on MMAs whose operands were loaded before it.
#pragma once

constexpr int kA4Threads = 384;
constexpr int kA4QStages = 1;
constexpr int kA4KStages = 3;
constexpr int kA4VStages = 3;
constexpr int kA4Prefetch = 4;  // key tiles ahead whose K/V boxes are prefetched into L2
// Q[1] | K[3] | V[3] | barriers + queue + partial row sums
constexpr int kA4BarOff = (kA4QStages + kA4KStages + kA4VStages) * kTileBytes;
constexpr int kA4Smem = kA4BarOff + 2048 + 1024;
constexpr int kA4RegsLow = 72;    // warps 0-3 after setmaxnreg.dec
constexpr int kA4RegsHigh = 216;  // warps 4-11 after setmaxnreg.inc (72*128 + 216*256 = 168*384)
static_assert(kA4RegsLow * 128 + kA4RegsHigh * 256 <= 168 * kA4Threads, "register split exceeds the launch");

enum : int {
  kB4QFull = 0,            // [2] (kA4QStages <= 2)
  kB4QEmpty = 2,           // [2]
  kB4KFull = 4,            // [3]
  kB4KEmpty = 7,           // [3]
  kB4VFull = 10,           // [3]
  kB4VEmpty = 13,          // [3]
  kB4SFull = 16,           // [2] S(t) in TMEM
  kB4SFree = 18,           // [2] softmax has read S(t)            (count 256)
  kB4PFull = 20,           // [2] P(t) written, O rescaled         (count 256)
  kB4PFree = 22,           // [2] PV(t) complete
  kB4OFull = 24,           // last PV of the item complete
  kB4OFree = 25,           // epilogue has read O                  (count 256)
  kB4ItFull = 26,          // [2]
  kB4ItEmpty = 28,         // [2]                                  (count 258)
  kB4Drain = 30,
  kB4LFull = 31,           // both halves of the row sums written  (count 256)
  kB4LFree = 32,           // both halves read                     (count 256)
  kB4Drain2 = 33,
  kB4Count = 34
};
static_assert(kA4QStages <= 2 && kA4KStages <= 3 && kA4VStages <= 3, "barrier layout");

// L2 prefetch of one TMA box (no shared-memory destination, no barrier)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// bounded wait used only while draining after an abort (no error recorded)
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
}

// a value the compiler must recompute where it is used (keeps MMA descriptors
// out of registers between uses instead of hoisting all of them)
__device__ __forceinline__ uint64_t opaque64(uint64_t v) {
  uint64_t r;
  asm volatile("mov.b64 %0, %1;" : "=l"(r) : "l"(v));
  return r;
}

__device__ __forceinline__ int item_tiles(const WorkItem& it) { return it.n_implicit + it.list_len; }

__device__ __forceinline__ void reg_dealloc4() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kA4RegsLow));
}
__device__ __forceinline__ void reg_alloc4() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kA4RegsHigh));
}

template <int POLY>
__global__ void __launch_bounds__(kA4Threads, 1)
    flash_attn4_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, AttnParams p, int n_items,
                       int* __restrict__ item_counter) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  auto sQ = [&](int b) { return sbase + (uint32_t)b * kTileBytes; };
  auto sK = [&](int s) { return sbase + (uint32_t)(kA4QStages + s) * kTileBytes; };
  auto sV = [&](int s) { return sbase + (uint32_t)(kA4QStages + kA4KStages + s) * kTileBytes; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kA4BarOff);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  volatile int* queue = reinterpret_cast<volatile int*>(bars + 40);  // [2] (barriers use bars[0, kB4Count))
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 41);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lsum = reinterpret_cast<float*>(bars + 64);  // [2][128] partial row sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kB4Count; ++i) {
      uint32_t c = 1;
      if (i == kB4SFree || i == kB4SFree + 1 || i == kB4PFull || i == kB4PFull + 1 || i == kB4OFree ||
          i == kB4LFull || i == kB4LFree)
        c = 256;
      if (i == kB4ItEmpty || i == kB4ItEmpty + 1) c = 258;
      mbar_init(bar(i), c);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    reg_dealloc4();
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      bool ok = true;
      uint32_t published = 0, nq = 0, nk = 0, nv = 0;
      auto publish = [&]() -> int {
        const uint32_t k = published;
        if (!mbar_wait(bar(kB4ItEmpty + (k & 1)), ((k >> 1) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
          ok = false;
          return -1;
        }
        int idx = atomicAdd(item_counter, 1);
        if (idx >= n_items) idx = -1;
        queue[k & 1] = idx;
        mbar_arrive(bar(kB4ItFull + (k & 1)));
        published = k + 1;
        if (idx >= 0) {  // warm L2 with the Q tile of the item after the current one
          const WorkItem w = p.items[idx];
          for (int ch = 0; ch < 2; ++ch)
            for (int rh = 0; rh < 2; ++rh) tma_prefetch_2d(&tmQ, w.head * 128 + ch * 64, w.q_start + rh * 64);
        }
        return idx;
      };
      auto load_kv = [&](const CUtensorMap* tm, uint32_t dst, uint32_t full, uint32_t empty, uint32_t par,
                         int hcol, int4 e) -> bool {
        if (!mbar_wait(empty, par, p.err, kDevTimeoutEmpty, abort_flag)) return false;
        mbar_arrive_expect_tx(full, kTileBytes);
        for (int ch = 0; ch < 2; ++ch) {
          tma_load_2d(dst + ch * 16384, tm, full, hcol + ch * 64, e.x);
          tma_load_2d(dst + ch * 16384 + 8192, tm, full, hcol + ch * 64, e.y);
        }
        return true;
      };
      auto load_k = [&](const WorkItem& it, int j) -> bool {
        const uint32_t s = nk % kA4KStages, par = ((nk / kA4KStages) & 1) ^ 1u;
        const bool r = load_kv(&tmK, sK(s), bar(kB4KFull + s), bar(kB4KEmpty + s), par, it.head * 128,
                               kv_entry(it, p.entries, j));
        ++nk;
        return r;
      };
      auto load_v = [&](const WorkItem& it, int j) -> bool {
        const uint32_t s = nv % kA4VStages, par = ((nv / kA4VStages) & 1) ^ 1u;
        const bool r = load_kv(&tmV, sV(s), bar(kB4VFull + s), bar(kB4VEmpty + s), par, it.head * 128,
                               kv_entry(it, p.entries, j));
        ++nv;
        return r;
      };
      int next = publish();
      while (ok && next >= 0) {
        const WorkItem it = p.items[next];
        next = publish();
        if (!ok) break;
        const int n = item_tiles(it);
        if (n == 0) continue;
        const uint32_t b = nq % kA4QStages;
        if (!mbar_wait(bar(kB4QEmpty + b), ((nq / kA4QStages) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar(kB4QFull + b), kTileBytes);
        for (int ch = 0; ch < 2; ++ch)
          for (int rh = 0; rh < 2; ++rh)
            tma_load_2d(sQ(b) + ch * 16384 + rh * 8192, &tmQ, bar(kB4QFull + b), it.head * 128 + ch * 64,
                        it.q_start + rh * 64);
        ++nq;
        if (!load_k(it, 0) || (n > 1 && !load_k(it, 1))) {
          ok = false;
          break;
        }
        for (int t = 0; t < n && ok; ++t) {
          if (t + 2 < n && !load_k(it, t + 2)) ok = false;
          if (ok && !load_v(it, t)) ok = false;
          if (t + 2 + kA4Prefetch < n) {  // warm L2 for the loads a few tiles ahead
            const int4 e = kv_entry(it, p.entries, t + 2 + kA4Prefetch);
            for (int ch = 0; ch < 2; ++ch) {
              tma_prefetch_2d(&tmK, it.head * 128 + ch * 64, e.x);
              tma_prefetch_2d(&tmK, it.head * 128 + ch * 64, e.y);
              tma_prefetch_2d(&tmV, it.head * 128 + ch * 64, e.x);
              tma_prefetch_2d(&tmV, it.head * 128 + ch * 64, e.y);
            }
          }
        }
      }
      if (!ok) {  // let copies already issued land before the CTA exits
        for (uint32_t i = nq > kA4QStages ? nq - kA4QStages : 0; i < nq; ++i)
          mbar_drain(bar(kB4QFull + i % kA4QStages), (i / kA4QStages) & 1);
        for (uint32_t i = nk > kA4KStages ? nk - kA4KStages : 0; i < nk; ++i)
          mbar_drain(bar(kB4KFull + i % kA4KStages), (i / kA4KStages) & 1);
        for (uint32_t i = nv > kA4VStages ? nv - kA4VStages : 0; i < nv; ++i)
          mbar_drain(bar(kB4VFull + i % kA4VStages), (i / kA4VStages) & 1);
      }
    }
  } else if (warp == 1 || warp == 2) {
    reg_dealloc4();
    // Two MMA issuers: one thread cannot issue tcgen05.mma much faster than one
    // per ~50 cycles, and a 128x128x16 MMA runs in 64, so a single issuer that
    // also waits on barriers starves the tensor pipe. Warp 1 issues S = Q K^T,
    // warp 2 issues O += P V; each commit tracks only its own thread's MMAs.
    if (lane == 0) {
      const bool s_role = warp == 1;
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);  // A = P from TMEM, B = V MN-major
      bool ok = true, issued = false;
      uint32_t taken = 0, nq = 0, nk = 0, nv = 0, g = 0, items_done = 0;
      while (ok) {
        const uint32_t k = taken;
        if (!mbar_wait(bar(kB4ItFull + (k & 1)), (k >> 1) & 1, p.err, kDevTimeoutFull, abort_flag)) break;
        const int idx = queue[k & 1];
        mbar_arrive(bar(kB4ItEmpty + (k & 1)));
        taken = k + 1;
        if (idx < 0) break;
        const int n = item_tiles(p.items[idx]);
        if (n == 0) continue;
        if (s_role) {
          const uint32_t qb = nq % kA4QStages;
          if (!mbar_wait(bar(kB4QFull + qb), (nq / kA4QStages) & 1, p.err, kDevTimeoutFull, abort_flag)) break;
          ++nq;
          const uint64_t dq = opaque64(smem_desc_sw128(sQ(qb), 16, 1024));
          for (int t = 0; t < n; ++t) {
            const uint32_t gt = g + t, b = gt & 1;
            // S buffer b was read (into registers) by the softmax of tile gt-2
            if (gt >= 2 &&
                !mbar_wait(bar(kB4SFree + b), ((gt >> 1) - 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t st = nk % kA4KStages;
            if (!mbar_wait(bar(kB4KFull + st), (nk / kA4KStages) & 1, p.err, kDevTimeoutFull, abort_flag)) {
              ok = false;
              break;
            }
            ++nk;
            tc_fence_after();
            const uint64_t dk = opaque64(smem_desc_sw128(sK(st), 16, 1024));
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
              umma_bf16(tmem + b * 128, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
            }
            issued = true;
            umma_commit(bar(kB4SFull + b));
            umma_commit(bar(kB4KEmpty + st));
            if (t == n - 1) umma_commit(bar(kB4QEmpty + qb));
          }
        } else {
          for (int t = 0; t < n; ++t) {
            const uint32_t gt = g + t, b = gt & 1;
            const uint32_t st = nv % kA4VStages;
            if (!mbar_wait(bar(kB4PFull + b), (gt >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag) ||
                !mbar_wait(bar(kB4VFull + st), (nv / kA4VStages) & 1, p.err, kDevTimeoutFull, abort_flag) ||
                (t == 0 && items_done > 0 &&
                 !mbar_wait(bar(kB4OFree), (items_done - 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag))) {
              ok = false;
              break;
            }
            ++nv;
            tc_fence_after();
            const uint64_t dv = opaque64(smem_desc_sw128(sV(st), 16384, 1024));
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16_ts(tmem + 384, tmem + 256 + b * 64 + kk * 8, dv + (uint64_t)(kk * (2048 >> 4)), idesc_o,
                           (t > 0 || kk > 0) ? 1u : 0u);
            issued = true;
            umma_commit(bar(kB4PFree + b));
            umma_commit(bar(kB4VEmpty + st));
          }
          if (ok) {
            umma_commit(bar(kB4OFull));
            ++items_done;
          }
        }
        g += n;
      }
      if (issued) {  // every MMA of this thread completes before TMEM is released
        const uint32_t d = bar(s_role ? kB4Drain : kB4Drain2);
        umma_commit(d);
        mbar_drain(d, 0);
      }
    }
  } else if (warp == 3) {
    reg_dealloc4();
  } else {
    reg_alloc4();
    // ------------------------------------------------ softmax + epilogue (2 warpgroups)
    const int w = (warp - 4) >> 2;  // column half of every tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qh = r >> 6;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_addr + 384 + (uint32_t)(w * 64);
    bool ok = true;
    uint32_t taken = 0, g = 0, items_done = 0, ep = 0;
    while (ok) {
      const uint32_t k = taken;
      if (!mbar_wait(bar(kB4ItFull + (k & 1)), (k >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
      const int idx = queue[k & 1];
      mbar_arrive(bar(kB4ItEmpty + (k & 1)));
      taken = k + 1;
      if (idx < 0) break;
      const WorkItem it = p.items[idx];
      const int n_kv = item_tiles(it);
      float m = -INFINITY;
      float l = 0.f;  // this warpgroup's half of the row sum
      int4 e = n_kv > 0 ? kv_entry(it, p.entries, 0) : make_int4(0, 0, 0, 0);
      for (int t = 0; t < n_kv; ++t) {
        const uint32_t gt = g + t, b = gt & 1;
        const int4 cur = e;
        if (t + 1 < n_kv) e = kv_entry(it, p.entries, t + 1);
        if (!mbar_wait(bar(kB4SFull + b), (gt >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // own half h = key columns [64w, 64w+64), other half x: both for the row max
        float h[64], x[64];
        const uint32_t tS = tmem + lane_addr + b * 128;
        tmem_ld32(tS + w * 64, *reinterpret_cast<float(*)[32]>(h));
        tmem_ld32(tS + w * 64 + 32, *reinterpret_cast<float(*)[32]>(h + 32));
        tmem_ld32(tS + (w ^ 1) * 64, *reinterpret_cast<float(*)[32]>(x));
        tmem_ld32(tS + (w ^ 1) * 64 + 32, *reinterpret_cast<float(*)[32]>(x + 32));
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(bar(kB4SFree + b));  // S(t) is in registers: S(t+2) may overwrite it
        const int lim0 = ((cur.z >> (8 + qh)) & 1) ? (cur.z & 0xFF) : 0;
        const int lim1 = ((cur.w >> (8 + qh)) & 1) ? (cur.w & 0xFF) : 0;
        if (__any_sync(0xffffffffu, lim0 != 64 || lim1 != 64)) {
          const int limh = w == 0 ? lim0 : lim1, limx = w == 0 ? lim1 : lim0;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            if (i >= limh) h[i] = -INFINITY;
            if (i >= limx) x[i] = -INFINITY;
          }
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          mx[0] = max3f(mx[0], h[i], h[i + 1]);
          mx[1] = max3f(mx[1], h[i + 2], h[i + 3]);
          mx[2] = max3f(mx[2], x[i], x[i + 1]);
          mx[3] = max3f(mx[3], x[i + 2], x[i + 3]);
        }
        const float m_new = fmaxf(m, max3f(fmaxf(mx[0], mx[1]), mx[2], mx[3]));
        bool need = false;
        if (t == 0) {
          m = m_new;
        } else {
          need = (m_new - m) * p.sl2 > 8.0f;
        }
        const bool any_need = __any_sync(0xffffffffu, need);
        float alpha = 1.0f;
        if (need) {
          alpha = ex2((m - m_new) * p.sl2);
          m = m_new;
        }
        const float mu = (m == -INFINITY) ? 0.f : m * p.sl2;
        const float2 sl2x2 = make_float2(p.sl2, p.sl2);
        const float2 nmu2 = make_float2(-mu, -mu);
        // P(t) buffer b was last read by PV(t-2)
        if (gt >= 2) {
          if (!mbar_wait(bar(kB4PFree + b), ((gt >> 1) - 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
            ok = false;
            break;
          }
        }
        float2 rs2[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) rs2[q] = make_float2(0.f, 0.f);
        const uint32_t tP = tmem + lane_addr + 256 + b * 64 + (uint32_t)(w * 32);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = 32 * c + 2 * i;
            const float2 a = __ffma2_rn(make_float2(h[col], h[col + 1]), sl2x2, nmu2);
            float2 pv;
            if ((i & 3) < POLY) {
              pv = ex2_poly2(a);
            } else {
              pv = make_float2(ex2(a.x), ex2(a.y));
            }
            rs2[i & 3] = __fadd2_rn(rs2[i & 3], pv);
            pk[i] = pack_bf16x2(pv.x, pv.y);
          }
          tmem_st16(tP + c * 16, pk);
        }
        if (any_need) {
          // O is accumulated by PV(t-1): wait for it, then rescale this half in place
          if (t >= 1 && !mbar_wait(bar(kB4PFree + (b ^ 1)), ((gt - 1) >> 1) & 1, p.err, kDevTimeoutSoftmax,
                                   abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
        tmem_wait_st();
        {
          const float2 a = __fadd2_rn(rs2[0], rs2[1]), c2 = __fadd2_rn(rs2[2], rs2[3]);
          const float2 u = __fadd2_rn(a, c2);
          l = l * alpha + (u.x + u.y);
        }
        tc_fence_before();
        mbar_arrive(bar(kB4PFull + b));
      }
      if (!ok) break;
      g += n_kv;
      // ---- epilogue: row sum = both halves; O half / l (with the SOL tail term)
      // (bounded mbarrier waits instead of a named barrier: an aborting thread
      // must not leave the others waiting forever)
      if (ep > 0 && !mbar_wait(bar(kB4LFree), (ep - 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
      lsum[w * 128 + r] = l;
      mbar_arrive(bar(kB4LFull));
      if (!mbar_wait(bar(kB4LFull), ep & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
      const float lrow = l + lsum[(w ^ 1) * 128 + r];
      mbar_arrive(bar(kB4LFree));
      ++ep;
      if (n_kv > 0) {
        if (!mbar_wait(bar(kB4OFull), items_done & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
        ++items_done;
        tc_fence_after();
      }
      const int ti = qh == 0 ? it.tail0 : it.tail1;
      float a1 = 1.f, a2 = 0.f, lt = lrow;
      const float* T = nullptr;
      const float ms = m * p.sl2;
      if (p.tailT && ti >= 0) {
        const int64_t o = (int64_t)it.head * p.nqb + ti;
        const float C2 = p.tailC[o] * 1.4426950408889634f;
        if (C2 > -INFINITY) {
          const float M2 = fmaxf(ms, C2);
          a1 = (m == -INFINITY) ? 0.f : ex2(ms - M2);
          a2 = ex2(C2 - M2);
          lt = lrow * a1 + p.tailL[o] * a2;
          T = p.tailT + o * 128 + w * 64;
        }
      }
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      const bool row_ok = r < it.q_rows;
      __nv_bfloat16* orow = p.out + (int64_t)(it.q_start + r) * p.out_stride + it.head * 128 + w * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float o[32];
        if (n_kv > 0) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (T) {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = o[i] * a1 + T[c * 32 + i] * a2;
        }
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8)
            *reinterpret_cast<uint4*>(orow + c * 32 + i) =
                make_uint4(pack_bf16x2(o[i] * inv, o[i + 1] * inv), pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv),
                           pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv), pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv));
        }
      }
      if (n_kv > 0) {
        tc_fence_before();
        mbar_arrive(bar(kB4OFree));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
