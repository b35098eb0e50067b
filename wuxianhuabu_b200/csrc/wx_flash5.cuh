// wx_flash5.cuh — flash-attention kernel for PAIRS of query tiles that walk the
// same key tiles (strip rows and dense layers: every key of the sequence), so
// each K/V tile is loaded once for 256 query rows (included by wx_attn.cu after
// wx_flash.cuh, whose helpers it shares). Head dimension HD = 128 (the H3 and
// benchmark geometries) or 64 (benchmark config 1).
//
// One CTA per pair (head, q tiles A and B). Per key tile t the tensor pipe runs
// S_X = Q_X K^T and O_X += P_X V for X in {A, B} (2048 cycles at HD 128); the
// shared K/V tile halves the load traffic per FLOP of a single-tile kernel.
//   TMEM (512 columns): S/P_A [0,128), S/P_B [128,256), O_A [256,256+HD),
//   O_B [384,384+HD); P_X overwrites the first 64 columns of S_X as packed bf16.
//   Shared memory: Q_A, Q_B, K ring of 3, V ring of 2 (128 x HD bf16 tiles, SW128,
//   in 64-column chunks).
//   Warp 0: TMA producer. Warp 1 / warp 2: MMA issuer of slot A / B (one
//   thread each: S_X(t), then PV_X(t) in four pieces of 32 keys, each issued as
//   soon as the softmax has stored that piece of P_X(t), then S_X(t+1) — the
//   tensor pipe runs one thread's MMAs in issue order, so S_X(t+1) cannot
//   overwrite P_X(t) before PV_X(t) has read it). Warp 3: idle.
//   Warps 4-7 / 8-11: softmax + epilogue of slot A / B (thread r owns row r).
//   (DUO: warp 3 loads V while warp 0 loads Q and K.)
// The exponential phases of the two slots' softmaxes take turns (A(t) after
// B(t-1), B(t) after A(t)); the TMEM loads and row max of one slot overlap the
// exponentials of the other, and the tensor pipe runs PV and the next S meanwhile.
//
// DUO = true runs the same schedule for two INDEPENDENT work items (the routed
// video query tiles, whose key lists differ): each slot streams its own K and V
// (one buffer each: Q_A, Q_B, K_A, V_A, K_B, V_B), slots may have different tile
// counts (the turn is not awaited from a slot that has finished), and the
// epilogue adds the SOL tail term.
#pragma once

constexpr int kA5KStages = 3;
constexpr int kA5VStages = 2;
#ifndef WX_A5_TURN_CHUNK
#define WX_A5_TURN_CHUNK 3
#endif
constexpr int kA5TurnChunk = WX_A5_TURN_CHUNK;  // exponential chunks (of 4) after which the turn passes
// P(t) is handed to the MMA issuer in kA5PVParts pieces (of the 4 chunks of 32 keys): the
// PV(t) MMAs of a piece go out while the softmax still computes the next piece
#ifndef WX_A5_PV_PARTS
#define WX_A5_PV_PARTS 4
#endif
constexpr int kA5PVParts = WX_A5_PV_PARTS;
// Paired (shared K/V) mode: S(t+1) in two halves of 64 keys. Keys 64..127 land in S
// columns [64,128), which P(t) (bf16 in columns [0,64)) does not use, so that half
// is issued as soon as the softmax has read S(t); only keys 0..63 wait for PV(t).
#ifndef WX_A5_S_SPLIT
#define WX_A5_S_SPLIT 0
#endif
constexpr bool kA5SSplit = WX_A5_S_SPLIT != 0;
static_assert(kA5PVParts == 1 || kA5PVParts == 2 || kA5PVParts == 4, "P pieces: 1, 2 or 4");
// shared-memory plan of the kernel for head dimension HD
template <int HD>
struct A5Geom {
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static constexpr int kTile = 128 * HD * 2;  // one 128-row Q, K or V tile
  static constexpr int kChunks = HD / 64;     // 64-column SW128 chunks per tile
  static constexpr int kBarOff = (2 + kA5KStages + kA5VStages) * kTile;
  static constexpr int kSmem = kBarOff + 512 + 1024;
};

enum : int {
  kB5QFull = 0,
  kB5KFull = 1,   // [3]
  kB5KEmpty = 4,  // [3] count 2 (both slots' S)
  kB5VFull = 7,   // [2]
  kB5VEmpty = 9,  // [2] count 2 (both slots' PV)
  kB5SFull = 11,  // [2] per slot
  kB5PFull = 13,  // [2][kA5PVParts] per slot and piece of P, count 4 (one per softmax warp)
  kB5OFull = 13 + 2 * kA5PVParts,  // [2] per slot
  kB5Drain = kB5OFull + 2,         // [2] per slot
  kB5Turn = kB5Drain + 2,          // [2] per slot, count 4: this slot's exponentials (all but the tail) are issued
  kB5SRead = kB5Turn + 2,          // [2] per slot, count 4: the softmax has read S(t) into registers
  kB5Count = kB5SRead + 2
};
static_assert(kB5Count <= 32, "barriers overlap the TMEM slot");

template <bool DUO, int HD>
__global__ void __launch_bounds__(kA5Threads, 1)
    flash_attn_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, AttnParams p, int n_items) {
  using G = A5Geom<HD>;
  constexpr int kTile = G::kTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  auto sQ = [&](int X) { return sbase + (uint32_t)X * kTile; };
  // shared K ring / V ring, or (DUO) K_X at tile 2 + 2X and V_X at tile 3 + 2X
  auto sK = [&](int s) { return sbase + (uint32_t)(2 + s) * kTile; };
  auto sV = [&](int s) { return sbase + (uint32_t)((DUO ? 3 : 2 + kA5KStages) + s) * kTile; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kBarOff);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the pair: items 2b and 2b+1 (shared mode: same head and key stream; DUO: any two
  // items, the second absent when n_items is odd)
  const bool has_b = 2 * (int)blockIdx.x + 1 < n_items;
  const WorkItem itA = p.items[2 * blockIdx.x];
  const int nA = item_tiles(itA);
  const int nB = has_b ? item_tiles(p.items[2 * blockIdx.x + 1]) : 0;
  const int n_kv = DUO ? (nA > nB ? nA : nB) : nA;  // tiles of the longer slot
  const int hcol = itA.head * HD;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kB5Count; ++i) {
      uint32_t c = 1;
      if (!DUO && (i == kB5KEmpty || i == kB5KEmpty + 1 || i == kB5KEmpty + 2 || i == kB5VEmpty || i == kB5VEmpty + 1))
        c = 2;
      if ((i >= kB5PFull && i < kB5PFull + 2 * kA5PVParts) || i == kB5Turn || i == kB5Turn + 1 ||
          i == kB5SRead || i == kB5SRead + 1)
        c = 4;  // one per softmax warp
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
    reg_dealloc_low();
    if (lane == 0 && n_kv > 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      bool ok = true;
      uint32_t nk = 0, nv = 0, nk_b = 0;  // loads issued (DUO: K of slot A, K of slot B)
      const int nslots = (DUO && !has_b) ? 1 : 2;
      mbar_arrive_expect_tx(bar(kB5QFull), nslots * kTile);
      for (int X = 0; X < nslots; ++X) {
        const WorkItem w = p.items[2 * blockIdx.x + X];
        for (int ch = 0; ch < G::kChunks; ++ch)
          for (int rh = 0; rh < 2; ++rh)
            tma_load_2d(sQ(X) + ch * kChunkBytes + rh * kHalfBytes, &tmQ, bar(kB5QFull), w.head * HD + ch * 64,
                        w.q_start + rh * 64);
      }
      auto tile_load = [&](const CUtensorMap* tm, uint32_t dst, uint32_t full, int hc, int4 e) {
        mbar_arrive_expect_tx(full, kTile);
        for (int ch = 0; ch < G::kChunks; ++ch) {
          tma_load_2d(dst + ch * kChunkBytes, tm, full, hc + ch * 64, e.x);
          tma_load_2d(dst + ch * kChunkBytes + kHalfBytes, tm, full, hc + ch * 64, e.y);
        }
      };
      if constexpr (!DUO) {
        auto load = [&](bool is_k, int j) -> bool {
          const uint32_t cnt = is_k ? nk : nv;
          const int ns = is_k ? kA5KStages : kA5VStages;
          const uint32_t s = cnt % ns, par = ((cnt / ns) & 1) ^ 1u;
          if (!mbar_wait(bar((is_k ? kB5KEmpty : kB5VEmpty) + s), par, p.err, kDevTimeoutEmpty, abort_flag))
            return false;
          tile_load(is_k ? &tmK : &tmV, is_k ? sK(s) : sV(s), bar((is_k ? kB5KFull : kB5VFull) + s), hcol,
                    kv_entry(itA, p, j));
          if (is_k) ++nk; else ++nv;
          return true;
        };
        // consumption order of each issuer: K(0), V(0), K(1), V(1), ... with the K
        // ring two tiles ahead of the V ring
        ok = load(true, 0) && (n_kv < 2 || load(true, 1));
        for (int t = 0; t < n_kv && ok; ++t) {
          ok = load(false, t);
          if (ok && t + 2 < n_kv) ok = load(true, t + 2);
        }
      } else {
        // one K buffer per slot: K_X(t) waits for S_X(t-1). The V loads come from warp 3
        // so that a slow V never holds back the next K.
        const WorkItem itB = p.items[2 * blockIdx.x + (has_b ? 1 : 0)];
        for (int t = 0; t < n_kv && ok; ++t) {
          for (int X = 0; X < 2 && ok; ++X) {
            if (t >= (X == 0 ? nA : nB)) continue;
            const WorkItem& w = X == 0 ? itA : itB;
            if (!mbar_wait(bar(kB5KEmpty + X), ((uint32_t)t & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
              ok = false;
              break;
            }
            tile_load(&tmK, sK(2 * X), bar(kB5KFull + X), w.head * HD, kv_entry(w, p, t));
            (X == 0 ? nk : nk_b) = (uint32_t)t + 1;
          }
        }
      }
      if (!ok) {  // let copies already issued land before the CTA exits
        mbar_drain(bar(kB5QFull), 0);
        if constexpr (!DUO) {
          for (uint32_t i = nk > kA5KStages ? nk - kA5KStages : 0; i < nk; ++i)
            mbar_drain(bar(kB5KFull + i % kA5KStages), (i / kA5KStages) & 1);
          for (uint32_t i = nv > kA5VStages ? nv - kA5VStages : 0; i < nv; ++i)
            mbar_drain(bar(kB5VFull + i % kA5VStages), (i / kA5VStages) & 1);
        } else {
          if (nk) mbar_drain(bar(kB5KFull), (nk - 1) & 1);
          if (nk_b) mbar_drain(bar(kB5KFull + 1), (nk_b - 1) & 1);
        }
      }
    }
  } else if (warp == 1 || warp == 2) {
    reg_dealloc_low();
    const int X = warp - 1;
    const int nX = X == 0 ? nA : nB;
    if (lane == 0 && nX > 0) {
      // ------------------------------------------------------------ MMA issuer of slot X
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, HD, false, true);  // A = P from TMEM, B = V MN-major
      const uint32_t tS = tmem + (uint32_t)(X * 128);
      const uint32_t tO = tmem + 256 + (uint32_t)(X * 128);
      bool ok = mbar_wait(bar(kB5QFull), 0, p.err, kDevTimeoutFull, abort_flag);
      bool issued = false;
      const uint64_t dq = opaque64(smem_desc_sw128(sQ(X), 16, 1024));
      // buffer, barrier offset and phase of K(t) / V(t) for this slot
      auto kbuf = [&](int t) { return DUO ? 2 * X : t % kA5KStages; };
      auto kpar = [&](int t) { return DUO ? ((uint32_t)t & 1) : (((uint32_t)t / kA5KStages) & 1); };
      auto kbar = [&](int t) { return DUO ? X : t % kA5KStages; };
      auto vbuf = [&](int t) { return DUO ? 2 * X : t % kA5VStages; };
      auto vpar = [&](int t) { return DUO ? ((uint32_t)t & 1) : (((uint32_t)t / kA5VStages) & 1); };
      auto vbar = [&](int t) { return DUO ? X : t % kA5VStages; };
      // S(t) into S/P_X; its K tile must have landed (k_full waited by the caller)
      auto issue_s = [&](int t) {
        tc_fence_after();
        const uint64_t dk = opaque64(smem_desc_sw128(sK(kbuf(t)), 16, 1024));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_bf16(tS, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit(bar(kB5SFull + X));
        umma_commit(bar(kB5KEmpty + kbar(t)));
      };
      // one half of S(t) (keys 64*half .. 64*half+63 into S columns [64*half, 64*half+64))
      constexpr uint32_t idesc_s64 = idesc_bf16_f32(128, 64, false, false);
      auto issue_s_half = [&](int t, int half) {
        tc_fence_after();
        const uint64_t dk = opaque64(smem_desc_sw128(sK(kbuf(t)) + (uint32_t)half * kHalfBytes, 16, 1024));
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_bf16(tS + (uint32_t)(half * 64), dq + off, dk + off, idesc_s64, kk > 0 ? 1u : 0u);
        }
        issued = true;
      };
      constexpr bool split = kA5SSplit && !DUO;
      auto k_ready = [&](int t) {
        return mbar_wait(bar(kB5KFull + kbar(t)), kpar(t), p.err, kDevTimeoutFull, abort_flag);
      };
      if (ok && (ok = k_ready(0))) issue_s(0);
      for (int t = 0; t < nX && ok; ++t) {
        // V(t) and K(t+1) are waited for before P(t): once the softmax hands over P(t),
        // PV(t) and S(t+1) go out back to back with no barrier wait between them
        if (!mbar_wait(bar(kB5VFull + vbar(t)), vpar(t), p.err, kDevTimeoutFull, abort_flag) ||
            (t + 1 < nX && !k_ready(t + 1))) {
          ok = false;
          break;
        }
        if (split && t + 1 < nX) {
          // keys 64..127 of S(t+1) as soon as the softmax has read S(t)
          if (!mbar_wait(bar(kB5SRead + X), (uint32_t)t & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
            ok = false;
            break;
          }
          issue_s_half(t + 1, 1);
        }
        const uint64_t dv = opaque64(smem_desc_sw128(sV(vbuf(t)), kChunkBytes, 1024));
        constexpr int kk_per = 8 / kA5PVParts;
#pragma unroll
        for (int part = 0; part < kA5PVParts && ok; ++part) {
          if (!mbar_wait(bar(kB5PFull + X * kA5PVParts + part), (uint32_t)t & 1, p.err, kDevTimeoutSoftmax,
                         abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k2 = 0; k2 < kk_per; ++k2) {
            const int kk = part * kk_per + k2;
            umma_bf16_ts(tO, tS + kk * 8, dv + (uint64_t)(kk * (2048 >> 4)), idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
          }
        }
        if (!ok) break;
        umma_commit(bar(kB5VEmpty + vbar(t)));
        if (t + 1 < nX) {
          if (split) {
            issue_s_half(t + 1, 0);
            umma_commit(bar(kB5SFull + X));
            umma_commit(bar(kB5KEmpty + kbar(t + 1)));
          } else {
            issue_s(t + 1);
          }
        }
      }
      if (ok) umma_commit(bar(kB5OFull + X));
      if (issued) {  // every MMA of this thread completes before TMEM is released
        umma_commit(bar(kB5Drain + X));
        mbar_drain(bar(kB5Drain + X), 0);
      }
    }
  } else if (warp == 3) {
    reg_dealloc_low();
    if (DUO && lane == 0 && n_kv > 0) {
      // ------------------------------------------------------------ V producer (DUO)
      // one V buffer per slot: V_X(t) waits for PV_X(t-1)
      bool ok = true;
      uint32_t nv_a = 0, nv_b = 0;
      const WorkItem itB = p.items[2 * blockIdx.x + (has_b ? 1 : 0)];
      for (int t = 0; t < n_kv && ok; ++t) {
        for (int X = 0; X < 2 && ok; ++X) {
          if (t >= (X == 0 ? nA : nB)) continue;
          const WorkItem& w = X == 0 ? itA : itB;
          if (!mbar_wait(bar(kB5VEmpty + X), ((uint32_t)t & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const int4 e = kv_entry(w, p, t);
          const uint32_t full = bar(kB5VFull + X), dst = sV(2 * X);
          mbar_arrive_expect_tx(full, kTile);
          for (int ch = 0; ch < G::kChunks; ++ch) {
            tma_load_2d(dst + ch * kChunkBytes, &tmV, full, w.head * HD + ch * 64, e.x);
            tma_load_2d(dst + ch * kChunkBytes + kHalfBytes, &tmV, full, w.head * HD + ch * 64, e.y);
          }
          (X == 0 ? nv_a : nv_b) = (uint32_t)t + 1;
        }
      }
      if (!ok) {
        if (nv_a) mbar_drain(bar(kB5VFull), (nv_a - 1) & 1);
        if (nv_b) mbar_drain(bar(kB5VFull + 1), (nv_b - 1) & 1);
      }
    }
  } else {
    reg_alloc_high();
    // ------------------------------------------------ softmax + epilogue of slot X
    const int X = (warp - 4) >> 2;
    const bool present = X == 0 || has_b;
    const WorkItem it = p.items[2 * blockIdx.x + (present ? X : 0)];
    const int nX = X == 0 ? nA : nB;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qh = r >> 6;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_addr + (uint32_t)(X * 128);
    const uint32_t tO = tmem + lane_addr + 256 + (uint32_t)(X * 128);
    float m = -INFINITY;
    float l = 0.f;
    bool ok = true;
    int4 e = nX > 0 ? kv_entry(it, p, 0) : make_int4(0, 0, 0, 0);
    for (int t = 0; t < nX; ++t) {
      const int4 cur = e;
      if (t + 1 < nX) e = kv_entry(it, p, t + 1);
      if (!mbar_wait(bar(kB5SFull + X), (uint32_t)t & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<float(*)[32]>(v + c * 32));
      tmem_wait_ld();
      if constexpr (kA5SSplit && !DUO) {  // S(t) is in registers: the next S may overwrite keys 64..127
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kB5SRead + X));
      }
      const int lim0 = ((cur.z >> (8 + qh)) & 1) ? (cur.z & 0xFF) : 0;
      const int lim1 = ((cur.w >> (8 + qh)) & 1) ? (cur.w & 0xFF) : 0;
      if (__any_sync(0xffffffffu, lim0 != 64 || lim1 != 64)) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if ((i & 63) >= ((i < 64) ? lim0 : lim1)) v[i] = -INFINITY;
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 128; i += 8) {
        mx[0] = max3f(mx[0], v[i], v[i + 1]);
        mx[1] = max3f(mx[1], v[i + 2], v[i + 3]);
        mx[2] = max3f(mx[2], v[i + 4], v[i + 5]);
        mx[3] = max3f(mx[3], v[i + 6], v[i + 7]);
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
      if constexpr (kA5PVParts > 1) {
        if (any_need) {
          // O_X is rescaled before any PV_X(t) MMA (they start with the first piece of P);
          // PV_X(t-1) completed before S_X(t) (in-order tensor pipe), so O_X is stable
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
      }
      // The exponential phases of the two slots take turns (A(0), B(0), A(1),
      // B(1), ...): run together they would share the MUFU pipe while the tensor
      // pipe idles; in turns, each overlaps the other slot's TMEM loads, row max,
      // PV and next S.
      // The turn passes when the other slot has stored its chunk kA5TurnChunk of P
      // (by default the last: the phases do not overlap; with P handed over in
      // pieces, passing it earlier measured slower).
      // (A slot whose partner has no tile at that index does not wait.)
      const bool turn = X == 0 ? (t == 0 || t - 1 >= nB ||
                                  mbar_wait(bar(kB5Turn + 1), ((uint32_t)t - 1) & 1, p.err, kDevTimeoutSoftmax,
                                            abort_flag))
                               : (t >= nA ||
                                  mbar_wait(bar(kB5Turn + 0), (uint32_t)t & 1, p.err, kDevTimeoutSoftmax, abort_flag));
      if (!turn) {
        ok = false;
        break;
      }
      const float mu = (m == -INFINITY) ? 0.f : m * p.sl2;
      const float2 sl2x2 = make_float2(p.sl2, p.sl2);
      const float2 nmu2 = make_float2(-mu, -mu);
      float2 rs2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) rs2[q] = make_float2(0.f, 0.f);
      // p = 2^(s*scale*log2e - m) as packed bf16 over the first 64 S columns (read above)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 a = __ffma2_rn(make_float2(v[32 * c + 2 * i], v[32 * c + 2 * i + 1]), sl2x2, nmu2);
          const float2 pv = make_float2(ex2(a.x), ex2(a.y));
          rs2[i & 3] = __fadd2_rn(rs2[i & 3], pv);
          pk[i] = pack_bf16x2(pv.x, pv.y);
        }
        tmem_st16(tS + c * 16, pk);
        if (c == kA5TurnChunk) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kB5Turn + X));
        }
        if constexpr (kA5PVParts > 1) {
          constexpr int per = 4 / kA5PVParts;
          if ((c + 1) % per == 0) {  // this piece of P is in TMEM: its PV MMAs may start
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kB5PFull + X * kA5PVParts + (c + 1) / per - 1));
          }
        }
      }
      if constexpr (kA5PVParts == 1) {
        if (any_need) {
          // PV_X(t-1) completed before S_X(t) (in-order tensor pipe): O_X is stable
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
        tmem_wait_st();
      }
      {
        const float2 a = __fadd2_rn(rs2[0], rs2[1]), c2 = __fadd2_rn(rs2[2], rs2[3]);
        const float2 u = __fadd2_rn(a, c2);
        l = l * alpha + (u.x + u.y);
      }
      if constexpr (kA5PVParts == 1) {
        tc_fence_before();
        __syncwarp();  // the warp's TMEM stores are complete: one arrival per warp (4, not 128 atomics)
        if (lane == 0) mbar_arrive(bar(kB5PFull + X));
      }
    }
    if (ok && nX > 0) ok = mbar_wait(bar(kB5OFull + X), 0, p.err, kDevTimeoutSoftmax, abort_flag);
    tc_fence_after();
    // epilogue: O / l (with the SOL tail term for routed items) -> bf16 rows
    const int ti = qh == 0 ? it.tail0 : it.tail1;
    float a1 = 1.f, a2 = 0.f, lt = l;
    const float* T = nullptr;
    if (DUO && p.tailT && ti >= 0) {
      const float ms = m * p.sl2;
      const int64_t o = (int64_t)it.head * p.nqb + ti;
      const float C2 = p.tailC[o] * 1.4426950408889634f;
      if (C2 > -INFINITY) {
        const float M2 = fmaxf(ms, C2);
        a1 = (m == -INFINITY) ? 0.f : ex2(ms - M2);
        a2 = ex2(C2 - M2);
        lt = l * a1 + p.tailL[o] * a2;
        T = p.tailT + o * HD;
      }
    }
    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
    const bool row_ok = ok && present && r < it.q_rows &&
                        WX_IN_BOUNDS(p.err, attn_row_ok(p, (int64_t)it.q_start + r));
    __nv_bfloat16* orow = attn_out_row<HD>(p, (int64_t)(it.q_start + r), it.head);
#pragma unroll 1
    for (int c = 0; c < HD / 32 && present; ++c) {
      float o[32];
      if (nX > 0) {
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
  }

  if (p.sig.counter) peer_signal_cta_done(p.sig);  // rows written to other GPUs: tell them
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
