// wx_flash.cuh — tcgen05 flash-attention kernel over per-(head, q tile) key-tile
// lists (included by wx_attn.cu).
//
// One CTA per work item = (head, 128-row query tile). Warp roles (192 threads):
//   warp 0      TMA producer: Q once, then K/V tiles into a 2-stage ring
//   warp 1      MMA issuer (one thread) and TMEM owner
//   warps 2..5  softmax: thread r owns query row r (TMEM lane r)
// TMEM (512 columns): S double buffer [0,128) [128,256), O accumulator [256,384).
// Shared memory: Q 32 KB, K/V 2 x 64 KB, P double buffer 2 x 32 KB (all SW128).
//
// Per key tile j the MMA thread issues S_{j+1} = Q K_{j+1}^T before waiting for
// P_j, then O += P_j V_j. P is double-buffered, and both P-ready signals and PV
// completions alternate between two barriers (so that no waiter can fall two
// phases behind), so softmax of tile j only waits for PV_{j-2} (the last
// reader of its P buffer) — and for PV_{j-1} only in the rare case that the
// running max grew by more than 2^8 and O must be rescaled (lazy rescaling:
// otherwise p = 2^(s - m_stale) <= 2^8 and the stale max is kept).
#pragma once

constexpr int kAttnThreads = 192;
constexpr int kTileBytes = 128 * 128 * 2;  // one 128x128 bf16 operand tile
// Q | K0 V0 | K1 V1 | P0 P1 | barriers
constexpr int kAttnBarOffset = 7 * kTileBytes;
constexpr int kAttnSmem = kAttnBarOffset + 256 + 1024;

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
  // peer_col + head*128; out_peer[0] == nullptr writes to `out`. sig.counter !=
  // nullptr: the last CTA of the call signals every rank (peer_signal_cta_done).
  __nv_bfloat16* out_peer[kMaxPeers];
  int64_t peer_rows;
  int peer_col;
  PeerSignal sig;
};

// destination of output row `row` (query row of the sequence) of head `head`
__device__ __forceinline__ __nv_bfloat16* attn_out_row(const AttnParams& p, int64_t row, int head) {
  if (p.out_peer[0] == nullptr) return p.out + row * p.out_stride + head * 128;
  const int64_t owner = row / p.peer_rows;
  __nv_bfloat16* base = p.out_peer[0];
#pragma unroll
  for (int r = 1; r < kMaxPeers; ++r)
    if (owner == r) base = p.out_peer[r];
  return base + (row - owner * p.peer_rows) * p.out_stride + p.peer_col + head * 128;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe for a pair of arguments: x = j + f with j = round(x) and
// f in [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted by least squares (in
// relative error, at Chebyshev nodes) with max relative error 7.8e-5 — far below
// the bf16 rounding P goes through — and j added to the exponent bits. Arguments
// are clamped at -125 so that masked (-inf) scores give a negligible 2^-125.
// Used for part of each row so that the MUFU pipe and the FMA pipe share the work.
// POLY (template argument of the kernel) = pairs of every 4 evaluated this way.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 magic = make_float2(12582912.f, 12582912.f);  // 1.5 * 2^23: rounds to an integer
  const float2 t = __fadd2_rn(x, magic);
  const float2 jf = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(jf, make_float2(-1.f, -1.f), x);
  float2 q = __ffma2_rn(make_float2(0.05508868396282196f, 0.05508868396282196f), f,
                        make_float2(0.24260404706001282f, 0.24260404706001282f));
  q = __ffma2_rn(q, f, make_float2(0.6932762265205383f, 0.6932762265205383f));
  q = __ffma2_rn(q, f, make_float2(0.9999289512634277f, 0.9999289512634277f));
  // bits(t) = 0x4B400000 + j, and 0x4B400000 << 23 vanishes mod 2^32
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// three-input max (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// key tile j of a work item: two 64-row halves (start row, valid length | q-half mask << 8)
__device__ __forceinline__ int4 kv_entry(const WorkItem& it, const int4* entries, int j) {
  if (j < it.n_implicit) {
    const int s0 = j * 128;
    return make_int4(s0, s0 + 64, max(0, min(64, it.implicit_end - s0)) | (3 << 8),
                     max(0, min(64, it.implicit_end - s0 - 64)) | (3 << 8));
  }
  return __ldg(entries + it.list_begin + (j - it.n_implicit));
}

template <int POLY>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  // operand addresses (shared window): Q, K[st], V[st], P[b]
  const uint32_t sQ = sbase;
  auto sK = [&](int st) { return sbase + (uint32_t)(1 + 2 * st) * kTileBytes; };
  auto sV = [&](int st) { return sbase + (uint32_t)(2 + 2 * st) * kTileBytes; };
  auto sP = [&](int b) { return sbase + (uint32_t)(5 + b) * kTileBytes; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAttnBarOffset);
  // q_full, k_full[2], k_empty[2], s_full[2], p_full[2], o_done[2], v_full[2], v_empty[2]
  const uint32_t q_full = smem_u32(bars + 0);
  auto k_full = [&](int i) { return smem_u32(bars + 1 + i); };
  auto k_empty = [&](int i) { return smem_u32(bars + 3 + i); };
  auto v_full = [&](int i) { return smem_u32(bars + 11 + i); };
  auto v_empty = [&](int i) { return smem_u32(bars + 13 + i); };
  auto s_full = [&](int i) { return smem_u32(bars + 5 + i); };
  auto p_full = [&](int i) { return smem_u32(bars + 7 + i); };
  auto o_done = [&](int i) { return smem_u32(bars + 9 + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const WorkItem it = p.items[blockIdx.x];
  const int n_kv = it.n_implicit + it.list_len;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full(i), 1);
      mbar_init(k_empty(i), 1);
      mbar_init(v_full(i), 1);
      mbar_init(v_empty(i), 1);
      mbar_init(s_full(i), 1);
      mbar_init(o_done(i), 1);
      mbar_init(p_full(i), 128);
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
  const int hcol = it.head * 128;

  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      for (int ch = 0; ch < 2; ++ch)
        for (int rh = 0; rh < 2; ++rh)
          tma_load_2d(sQ + ch * 16384 + rh * 8192, &tmQ, q_full, hcol + ch * 64, it.q_start + rh * 64);
      int4 e = kv_entry(it, p.entries, 0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const int4 cur = e;
        if (j + 1 < n_kv) e = kv_entry(it, p.entries, j + 1);
        // K of stage st is free once S_{j-2} is done, V once PV_{j-2} is done
        if (!mbar_wait(k_empty(st), ((j >> 1) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(k_full(st), kTileBytes);
        for (int ch = 0; ch < 2; ++ch) {
          const uint32_t ko = sK(st) + ch * 16384;
          tma_load_2d(ko, &tmK, k_full(st), hcol + ch * 64, cur.x);
          tma_load_2d(ko + 8192, &tmK, k_full(st), hcol + ch * 64, cur.y);
        }
        if (!mbar_wait(v_empty(st), ((j >> 1) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(v_full(st), kTileBytes);
        for (int ch = 0; ch < 2; ++ch) {
          const uint32_t vo = sV(st) + ch * 16384;
          tma_load_2d(vo, &tmV, v_full(st), hcol + ch * 64, cur.x);
          tma_load_2d(vo + 8192, &tmV, v_full(st), hcol + ch * 64, cur.y);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);  // B = V, MN-major
      bool ok = mbar_wait(q_full, 0, p.err, kDevTimeoutFull, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(k_full(st), (j >> 1) & 1, p.err, kDevTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t ka = sK(st);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tmem + st * 128, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(ka + off, 16, 1024),
                    idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full(st));
        umma_commit(k_empty(st));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        if (!mbar_wait(p_full(j & 1), (j >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
        if (!mbar_wait(v_full(j & 1), (j >> 1) & 1, p.err, kDevTimeoutFull, abort_flag)) break;
        tc_fence_after();
        const uint32_t va = sV(j & 1), pa = sP(j & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = smem_desc_sw128(pa + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(va + kk * 2048, 16384, 1024);
          umma_bf16(tmem + 256, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(o_done(j & 1));
        umma_commit(v_empty(j & 1));
      }
    }
  } else {
    // softmax / correction / epilogue: thread owns TMEM lane (= q row) r
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qh = r >> 6;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY;  // running max of raw scores (unscaled)
    float l = 0.f;
    bool ok = true;
    // PV_k completion k alternates barriers: wait(k) = o_done[k&1] phase (k>>1)&1
    auto wait_pv = [&](int k) -> bool {
      return mbar_wait(o_done(k & 1), (k >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag);
    };
    int4 e = n_kv > 0 ? kv_entry(it, p.entries, 0) : make_int4(0, 0, 0, 0);
    for (int j = 0; j < n_kv && ok; ++j) {
      const int4 cur = e;
      if (j + 1 < n_kv) e = kv_entry(it, p.entries, j + 1);
      const int b = j & 1;
      if (!mbar_wait(s_full(b), (j >> 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_addr + b * 128 + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = t[i];
      }
      tmem_wait_ld();
      const int lim0 = ((cur.z >> (8 + qh)) & 1) ? (cur.z & 0xFF) : 0;
      const int lim1 = ((cur.w >> (8 + qh)) & 1) ? (cur.w & 0xFF) : 0;
      if (__any_sync(0xffffffffu, lim0 != 64 || lim1 != 64)) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const bool valid = (c < 64) ? (c < lim0) : ((c - 64) < lim1);
          if (!valid) sv[c] = -INFINITY;
        }
      }
      // row max: four independent chains (one softmax warp per SMSP has no other warp to hide latency)
      float mx[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mx[k] = fmaxf(sv[2 * k], sv[2 * k + 1]);
#pragma unroll
      for (int c = 8; c < 128; c += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mx[k] = max3f(mx[k], sv[c + 2 * k], sv[c + 2 * k + 1]);
      }
      const float rmax = max3f(fmaxf(mx[0], mx[1]), mx[2], mx[3]);
      const float m_new = fmaxf(m, rmax);
      bool need = false;
      if (j == 0) {
        m = m_new;
      } else {
        need = (m_new - m) * p.sl2 > 8.0f;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O holds PV_0..PV_{j-1}: wait for the last of them, then rescale in TMEM
        if (!wait_pv(j - 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = need ? ex2((m - m_new) * p.sl2) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float t[32];
          tmem_ld32(tmem + lane_addr + 256 + c * 32, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] *= alpha;
          tmem_st32(tmem + lane_addr + 256 + c * 32, t);
        }
        tmem_wait_st();
        l *= alpha;
        if (need) m = m_new;
      }
      // P buffer b was last read by PV_{j-2}
      if (j >= 2) {
        if (!wait_pv(j - 2)) {
          ok = false;
          break;
        }
      }
      const float mu = (m == -INFINITY) ? 0.f : m * p.sl2;
      // p = 2^(s*scale*log2e - m*scale*log2e): packed fp32x2 FMA for the argument,
      // MUFU ex2, packed fp32x2 adds for the row sum
      const float2 sl2x2 = make_float2(p.sl2, p.sl2);
      const float2 nmu2 = make_float2(-mu, -mu);
      float2 rs2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) rs2[q] = make_float2(0.f, 0.f);
      const uint32_t prow = sP(b) + r * 128;
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        float pv[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 a = __ffma2_rn(make_float2(sv[cc * 8 + 2 * q], sv[cc * 8 + 2 * q + 1]), sl2x2, nmu2);
          if (q < POLY) {
            const float2 e2 = ex2_poly2(a);
            pv[2 * q] = e2.x;
            pv[2 * q + 1] = e2.y;
          } else {
            pv[2 * q] = ex2(a.x);
            pv[2 * q + 1] = ex2(a.y);
          }
          rs2[q] = __fadd2_rn(rs2[q], make_float2(pv[2 * q], pv[2 * q + 1]));
        }
        const int atom = cc >> 3, c8 = cc & 7;
        const uint32_t addr = prow + atom * 16384 + ((c8 ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pack_bf16x2(pv[0], pv[1])),
                     "r"(pack_bf16x2(pv[2], pv[3])), "r"(pack_bf16x2(pv[4], pv[5])), "r"(pack_bf16x2(pv[6], pv[7]))
                     : "memory");
      }
      {
        const float2 a = __fadd2_rn(rs2[0], rs2[1]), c2 = __fadd2_rn(rs2[2], rs2[3]);
        const float2 t = __fadd2_rn(a, c2);
        l += t.x + t.y;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full(b));
    }
    if (ok && n_kv > 0) ok = wait_pv(n_kv - 1);  // its commit covers every earlier MMA
    tc_fence_after();
    // epilogue: tail term, normalisation, bf16 store
    const int ti = qh == 0 ? it.tail0 : it.tail1;
    float a1 = 1.f, a2 = 0.f, lt = l;
    const float* T = nullptr;
    const float ms = m * p.sl2;  // running max in the exp2 domain
    if (p.tailT && ti >= 0) {
      const int64_t o = (int64_t)it.head * p.nqb + ti;
      const float C2 = p.tailC[o] * 1.4426950408889634f;
      if (C2 > -INFINITY) {
        const float M2 = fmaxf(ms, C2);
        a1 = (m == -INFINITY) ? 0.f : ex2(ms - M2);
        a2 = ex2(C2 - M2);
        lt = l * a1 + p.tailL[o] * a2;
        T = p.tailT + o * 128;
      }
    }
    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
    const bool row_ok = ok && r < it.q_rows;
    __nv_bfloat16* orow = p.out + (int64_t)(it.q_start + r) * p.out_stride + hcol;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float t[32];
      tmem_ld32(tmem + lane_addr + 256 + c * 32, t);
      tmem_wait_ld();
      if (n_kv == 0) {
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = 0.f;
      }
      if (T) {
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = t[i] * a1 + T[c * 32 + i] * a2;
      }
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 8)
          *reinterpret_cast<uint4*>(orow + c * 32 + i) =
              make_uint4(pack_bf16x2(t[i] * inv, t[i + 1] * inv), pack_bf16x2(t[i + 2] * inv, t[i + 3] * inv),
                         pack_bf16x2(t[i + 4] * inv, t[i + 5] * inv), pack_bf16x2(t[i + 6] * inv, t[i + 7] * inv));
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
