// wx_flash2.cuh — flash-attention kernel sized for TWO CTAs per SM, head_dim 128
// (included by wx_attn.cu after wx_flash.cuh, whose helpers it shares). It runs
// the routed (video) query tiles when the two-item kernel of wx_flash5.cuh is
// switched off (WX_ATTN_DUO=0) or its register split does not fit.
//
// The softmax of one (head, 128-row q tile) and the tensor-core work of another
// overlap because two CTAs share each SM, instead of two q tiles sharing one
// CTA: the kept key lists differ from q tile to q tile, so a CTA cannot share
// one K/V stream between two q tiles. Per CTA:
//   TMEM 256 columns: S [0,128) (P overwrites its first 64 columns as packed
//   bf16 once S is consumed), O [128,256).
//   Shared memory 96 KB: Q, K, V (one 128x128 bf16 tile each, SW128).
// Per key tile j: S_j = Q K_j^T (SS MMA) -> softmax reads S_j from TMEM in two
// passes (max, then exp) and writes P_j back into TMEM -> O += P_j V_j (TS MMA,
// A from TMEM). tcgen05.mma instructions of one thread run in issue order, so
// S_{j+1} (issued after PV_j) cannot overwrite P_j before PV_j has read it, and
// PV_{j-1} is complete whenever S_j is. K_{j+1} streams in once S_j is done, V_{j+1}
// once PV_j is done. Warp 0: TMA producer; warp 1: MMA issuer (one thread) and
// TMEM owner; warps 2-5: softmax and epilogue, thread r owning query row r.
#pragma once

constexpr int kA2Smem = 3 * kTileBytes + 256 + 1024;

__global__ void __launch_bounds__(kAttnThreads, 2)
    flash_attn2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + kTileBytes;
  const uint32_t sV = sQ + 2 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTileBytes);
  const uint32_t q_full = smem_u32(bars + 0);
  const uint32_t k_full = smem_u32(bars + 1);
  const uint32_t k_empty = smem_u32(bars + 2);
  const uint32_t v_full = smem_u32(bars + 3);
  const uint32_t v_empty = smem_u32(bars + 4);
  const uint32_t s_full = smem_u32(bars + 5);
  const uint32_t p_full = smem_u32(bars + 6);
  const uint32_t o_done = smem_u32(bars + 7);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const WorkItem it = p.items[blockIdx.x];
  const int n_kv = it.n_implicit + it.list_len;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);  // one arrival per softmax warp
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S/P: cols [0,128), O: [128,256)
  const int hcol = it.head * 128;

  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      for (int ch = 0; ch < 2; ++ch)
        for (int rh = 0; rh < 2; ++rh)
          tma_load_2d(sQ + ch * kChunkBytes + rh * kHalfBytes, &tmQ, q_full, hcol + ch * 64, it.q_start + rh * 64);
      int4 e = kv_entry(it, p, 0);
      for (int j = 0; j < n_kv; ++j) {
        const int4 cur = e;
        if (j + 1 < n_kv) e = kv_entry(it, p, j + 1);
        if (!mbar_wait(k_empty, (j & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(k_full, kTileBytes);
        for (int ch = 0; ch < 2; ++ch) {
          tma_load_2d(sK + ch * kChunkBytes, &tmK, k_full, hcol + ch * 64, cur.x);
          tma_load_2d(sK + ch * kChunkBytes + kHalfBytes, &tmK, k_full, hcol + ch * 64, cur.y);
        }
        if (!mbar_wait(v_empty, (j & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(v_full, kTileBytes);
        for (int ch = 0; ch < 2; ++ch) {
          tma_load_2d(sV + ch * kChunkBytes, &tmV, v_full, hcol + ch * 64, cur.x);
          tma_load_2d(sV + ch * kChunkBytes + kHalfBytes, &tmV, v_full, hcol + ch * 64, cur.y);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);  // A from TMEM (K-major), B = V MN-major
      bool ok = mbar_wait(q_full, 0, p.err, kDevTimeoutFull, abort_flag);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (!mbar_wait(k_full, j & 1, p.err, kDevTimeoutFull, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tmem, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024), idesc_s,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(k_empty);
        if (!mbar_wait(p_full, j & 1, p.err, kDevTimeoutSoftmax, abort_flag)) break;
        if (!mbar_wait(v_full, j & 1, p.err, kDevTimeoutFull, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(tmem + 128, tmem + kk * 8, smem_desc_sw128(sV + kk * 2048, 16384, 1024), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(v_empty);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qh = r >> 6;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY;
    float l = 0.f;
    bool ok = true;
    int4 e = n_kv > 0 ? kv_entry(it, p, 0) : make_int4(0, 0, 0, 0);
    for (int j = 0; j < n_kv && ok; ++j) {
      const int4 cur = e;
      if (j + 1 < n_kv) e = kv_entry(it, p, j + 1);
      if (!mbar_wait(s_full, j & 1, p.err, kDevTimeoutSoftmax, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int lim0 = ((cur.z >> (8 + qh)) & 1) ? (cur.z & 0xFF) : 0;
      const int lim1 = ((cur.w >> (8 + qh)) & 1) ? (cur.w & 0xFF) : 0;
      const bool full = !__any_sync(0xffffffffu, lim0 != 64 || lim1 != 64);
      // pass 1: row max
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_addr + c * 32, t);
        tmem_wait_ld();
        if (!full) {
          const int lim = c < 2 ? lim0 : lim1;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if ((c & 1) * 32 + i >= lim) t[i] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          mx[0] = max3f(mx[0], t[i], t[i + 1]);
          mx[1] = max3f(mx[1], t[i + 2], t[i + 3]);
          mx[2] = max3f(mx[2], t[i + 4], t[i + 5]);
          mx[3] = max3f(mx[3], t[i + 6], t[i + 7]);
        }
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
        // PV_{j-1} completed before S_j (in-order tensor pipe): O is stable
        const float alpha = need ? ex2((m - m_new) * p.sl2) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float t[32];
          tmem_ld32(tmem + lane_addr + 128 + c * 32, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] *= alpha;
          tmem_st32(tmem + lane_addr + 128 + c * 32, t);
        }
        tmem_wait_st();
        l *= alpha;
        if (need) m = m_new;
      }
      const float mu = (m == -INFINITY) ? 0.f : m * p.sl2;
      const float2 sl2x2 = make_float2(p.sl2, p.sl2);
      const float2 nmu2 = make_float2(-mu, -mu);
      float2 rs2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) rs2[q] = make_float2(0.f, 0.f);
      // pass 2: p = 2^(s*scale*log2e - m), written back as packed bf16 over consumed S columns
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_addr + c * 32, t);
        tmem_wait_ld();
        if (!full) {
          const int lim = c < 2 ? lim0 : lim1;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if ((c & 1) * 32 + i >= lim) t[i] = -INFINITY;
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 a = __ffma2_rn(make_float2(t[2 * i], t[2 * i + 1]), sl2x2, nmu2);
          const float2 pv = make_float2(ex2(a.x), ex2(a.y));
          rs2[i & 3] = __fadd2_rn(rs2[i & 3], pv);
          pk[i] = pack_bf16x2(pv.x, pv.y);
        }
        tmem_st16(tmem + lane_addr + c * 16, pk);  // P columns [16c, 16c+16): S chunk c/2, already read
      }
      tmem_wait_st();
      {
        const float2 a = __fadd2_rn(rs2[0], rs2[1]), c2 = __fadd2_rn(rs2[2], rs2[3]);
        const float2 t = __fadd2_rn(a, c2);
        l += t.x + t.y;
      }
      tc_fence_before();
      __syncwarp();  // the warp's TMEM stores are complete: one arrival per warp
      if (lane == 0) mbar_arrive(p_full);
    }
    // the last PV: o_done completes once per tile and every earlier PV precedes S_{n-1}
    if (ok && n_kv > 0) ok = mbar_wait(o_done, (n_kv - 1) & 1, p.err, kDevTimeoutSoftmax, abort_flag);
    tc_fence_after();
    const int ti = qh == 0 ? it.tail0 : it.tail1;
    float a1 = 1.f, a2 = 0.f, lt = l;
    const float* T = nullptr;
    const float ms = m * p.sl2;
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
    const bool row_ok = ok && r < it.q_rows && WX_IN_BOUNDS(p.err, attn_row_ok(p, (int64_t)it.q_start + r));
    __nv_bfloat16* orow = p.out + (int64_t)(it.q_start + r) * p.out_stride + hcol;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float t[32];
      tmem_ld32(tmem + lane_addr + 128 + c * 32, t);
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
    tmem_dealloc(tmem, 256);
  }
}
