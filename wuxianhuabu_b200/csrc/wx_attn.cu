// wx_attn.cu — SOL block-sparse self-attention (H3SolAttn.forward,
// 网络算子-稀疏注意力-SOL通用.swift:388-532) and dense SDPA on sm_100a.
//
// Pipeline per layer:
//   1. block statistics of the video segment (q/k centroids, v sums, lengths)
//   2. router: SOL tau (centred centroid scores vs a per-(head, q-block)
//      threshold, diagonal +-1 and sink forced) or top-k (diagonal + the
//      ceil(density*nb) best other blocks)
//   3. tail pooling: the unselected blocks of each (head, q-block) folded into
//      one (max score C, weight sum L, value vector T) triple
//   4. kept-list builder: per (head, 128-row q tile) a list of 128-key tiles,
//      each made of two 64-key halves with per-(q-half, key-half) masks
//   5. flash kernels (tcgen05): strip / dense query tiles in pairs that share
//      each K/V tile, routed video tiles two independent items per CTA (same
//      schedule); S = Q K^T and O += P V on the tensor cores with P and O in
//      TMEM; online softmax in registers with lazy rescaling; tail term and
//      normalisation in the epilogue. head_dim 128 or 64.
// The routing arithmetic uses a fixed fp32 operation order (explicit _rn
// intrinsics) so that its decisions are bit-identical to the CPU oracle.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>

#include <algorithm>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

struct WorkItem {
  int q_start, q_rows, tail0, tail1;
  int list_begin, list_len, n_implicit, implicit_end;
  int head, pad0, pad1, pad2;
};

// ------------------------------------------------------------ 1. statistics
// grid (nb, H), block hd: sequential sums over the block's real rows.
__global__ void block_stats_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                   const __nv_bfloat16* __restrict__ v, int64_t row_stride, int64_t S, int hd,
                                   int64_t g, int block, int nb, float* __restrict__ qc, float* __restrict__ kc,
                                   __nv_bfloat16* __restrict__ vsum, float* __restrict__ lens) {
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int64_t r0 = g + (int64_t)b * block;
  const int64_t r1 = min(r0 + block, S);
  const float len = (float)(r1 - r0);
  float aq = 0.f, ak = 0.f, av = 0.f;
  const int64_t col = (int64_t)h * hd + d;
  int64_t s = r0;
  for (; s + 8 <= r1; s += 8) {  // 8 rows' loads in flight, then the sums in row order
    float xq[8], xk[8], xv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t o = (s + u) * row_stride + col;
      xq[u] = __bfloat162float(q[o]);
      xk[u] = __bfloat162float(k[o]);
      xv[u] = __bfloat162float(v[o]);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      aq = __fadd_rn(aq, xq[u]);
      ak = __fadd_rn(ak, xk[u]);
      av = __fadd_rn(av, xv[u]);
    }
  }
  for (; s < r1; ++s) {
    const int64_t o = s * row_stride + col;
    aq = __fadd_rn(aq, __bfloat162float(q[o]));
    ak = __fadd_rn(ak, __bfloat162float(k[o]));
    av = __fadd_rn(av, __bfloat162float(v[o]));
  }
  const int64_t idx = ((int64_t)h * nb + b) * hd + d;
  if (qc) qc[idx] = __fdiv_rn(aq, len);
  kc[idx] = __fdiv_rn(ak, len);
  vsum[idx] = __float2bfloat16_rn(av);
  if (h == 0 && d == 0) lens[b] = len;
}

// grid H, block hd: kMean over blocks, centre in place, kcVar = mean(kcc^2)
__global__ void kcenter_kernel(float* __restrict__ kc, int nb, int hd, float* __restrict__ kvar) {
  const int h = blockIdx.x, d = threadIdx.x;
  float* base = kc + (int64_t)h * nb * hd + d;
  constexpr int U = 16;  // loads in flight per chain; the sums stay in block order
  float acc = 0.f;
  int b = 0;
  for (; b + U <= nb; b += U) {
    float x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = base[(int64_t)(b + u) * hd];
#pragma unroll
    for (int u = 0; u < U; ++u) acc = __fadd_rn(acc, x[u]);
  }
  for (; b < nb; ++b) acc = __fadd_rn(acc, base[(int64_t)b * hd]);
  const float mean = __fdiv_rn(acc, (float)nb);
  float vacc = 0.f;
  for (b = 0; b + U <= nb; b += U) {
    float x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = __fsub_rn(base[(int64_t)(b + u) * hd], mean);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      base[(int64_t)(b + u) * hd] = x[u];
      vacc = __fadd_rn(vacc, __fmul_rn(x[u], x[u]));
    }
  }
  for (; b < nb; ++b) {
    const float c = __fsub_rn(base[(int64_t)b * hd], mean);
    base[(int64_t)b * hd] = c;
    vacc = __fadd_rn(vacc, __fmul_rn(c, c));
  }
  kvar[(int64_t)h * hd + d] = __fdiv_rn(vacc, (float)nb);
}

// thread per (h, qb): thr = tau * sqrt(sum_d((qc*qc)*kvar) * scale^2 + 1e-6)
__global__ void thr_kernel(const float* __restrict__ qc, const float* __restrict__ kvar, int H, int nb, int hd,
                           float scale, float tau, float* __restrict__ thr) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)H * nb) return;
  const int h = (int)(i / nb);
  const float* qr = qc + i * hd;
  const float* kv = kvar + (int64_t)h * hd;
  float var = 0.f;
  for (int d = 0; d < hd; ++d) var = __fadd_rn(var, __fmul_rn(__fmul_rn(qr[d], qr[d]), kv[d]));
  thr[i] = __fmul_rn(tau, __fsqrt_rn(__fadd_rn(__fmul_rn(var, __fmul_rn(scale, scale)), 1e-6f)));
}

// grid (ceil(nb/32), ceil(nb/8), H), block 256 = 32 key blocks x 8 query blocks.
// cm = bf16(fma-chain(qc, kc) * scale); mode 1: SOL selection, mode 2: f32 scores.
// grid (ceil(nb/64), ceil(nb/64), H), block 256: a 64x64 tile of block scores per
// CTA, 4x4 per thread (register tiling), head_dim in chunks of 32 through shared
// memory. Every score keeps the sequential fp32 order over d (d = 0, 1, ...) of
// the reference restatement, so the decisions stay bit-exact.
__global__ void __launch_bounds__(256) score_kernel(const float* __restrict__ qc, const float* __restrict__ kc,
                                                    int nb, int hd, float scale, int mode,
                                                    const float* __restrict__ thr, int sink_start, int sink_end,
                                                    __nv_bfloat16* __restrict__ cm, uint8_t* __restrict__ sel,
                                                    float* __restrict__ scores) {
  constexpr int T = 64, DC = 32;
  __shared__ float qs[T][DC + 1];
  __shared__ float ks[T][DC + 1];
  const int h = blockIdx.z;
  const int qb0 = blockIdx.y * T, kb0 = blockIdx.x * T;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int d0 = 0; d0 < hd; d0 += DC) {
    __syncthreads();
    for (int i = threadIdx.x; i < T * DC; i += 256) {
      const int r = i / DC, d = i % DC;
      qs[r][d] = (qb0 + r < nb) ? qc[((int64_t)h * nb + qb0 + r) * hd + d0 + d] : 0.f;
      ks[r][d] = (kb0 + r < nb) ? kc[((int64_t)h * nb + kb0 + r) * hd + d0 + d] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < DC; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = qs[ty * 4 + i][d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = ks[tx + 16 * j][d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(qv[i], kv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qb = qb0 + ty * 4 + i;
    if (qb >= nb) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kb = kb0 + tx + 16 * j;
      if (kb >= nb) continue;
      const float sc = __fmul_rn(acc[i][j], scale);
      const __nv_bfloat16 c = __float2bfloat16_rn(sc);
      const int64_t idx = ((int64_t)h * nb + qb) * nb + kb;
      cm[idx] = c;
      if (mode == WX_SPARSE_SOL) {
        bool s2 = __bfloat162float(c) > thr[(int64_t)h * nb + qb];
        if (abs(qb - kb) <= 1) s2 = true;
        if (kb >= sink_start && kb < sink_end) s2 = true;
        sel[idx] = (uint8_t)s2;
      } else {
        scores[idx] = sc;
      }
    }
  }
}

// grid (nb, H), block 256: the `keep` best off-diagonal blocks of row (h, qb) in the
// order (score desc, block index asc), plus the diagonal. Scores become order-
// preserving 32-bit keys (-0 folded into +0, so equal floats get equal keys); a
// radix select over 4 digits of 8 bits finds the keep-th key T; every key > T is
// kept, and of the keys == T the lowest block indices, in order, fill the rest.
__device__ __forceinline__ uint32_t score_key(float x) {
  const uint32_t u = __float_as_uint(__fadd_rn(x, 0.0f));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(256) topk_select_kernel(const float* __restrict__ scores, int nb, int keep,
                                                          uint8_t* __restrict__ sel) {
  extern __shared__ uint32_t keys[];  // [nb]; 0 = not a candidate (diagonal / padding)
  __shared__ int hist[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need;
  __shared__ int s_wsum[8];
  const int qb = blockIdx.x, h = blockIdx.y;
  const float* row = scores + ((int64_t)h * nb + qb) * nb;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) keys[i] = (i == qb) ? 0u : score_key(row[i]);
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = keep;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0 && keep > 0; shift -= 8) {
    hist[threadIdx.x] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const uint32_t k = keys[i];
      if (k && (k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l owns bins [8l, 8l+8): find the bin where the count from the top reaches `need`
      const int lane = threadIdx.x;
      int local = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) local += hist[lane * 8 + b];
      int suf = local;  // inclusive suffix sum over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += v;
      }
      const int above = suf - local;  // candidates in the bins of lanes > lane
      const int need = s_need;
      const bool here = above < need && above + local >= need;  // exactly one lane
      if (here) {
        int cum = above;
        for (int b = 7; b >= 0; --b) {
          const int cnt = hist[lane * 8 + b];
          if (cum + cnt >= need) {
            s_prefix = prefix | ((uint32_t)(lane * 8 + b) << shift);
            s_need = need - cum;
            break;
          }
          cum += cnt;
        }
      }
      if (lane == 0) s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  // keys > T are kept; of keys == T the first s_need in index order
  const uint32_t T = s_prefix;
  const int need_eq = s_need;
  const int per = (nb + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(nb, i0 + per);
  int eq = 0;
  for (int i = i0; i < i1; ++i) eq += (keep > 0 && keys[i] == T && keys[i]) ? 1 : 0;
  // exclusive prefix of eq over threads (index order)
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = eq;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_wsum[wid] = incl;
  __syncthreads();
  int before = incl - eq;
  for (int w = 0; w < wid; ++w) before += s_wsum[w];
  uint8_t* srow = sel + ((int64_t)h * nb + qb) * nb;
  for (int i = i0; i < i1; ++i) {
    const uint32_t k = keys[i];
    bool keepit = (i == qb);
    if (keep > 0 && k) {
      if (k > T) {
        keepit = true;
      } else if (k == T) {
        keepit = before < need_eq;
        ++before;
      }
    }
    srow[i] = (uint8_t)keepit;
  }
}

// ------------------------------------------------------------- 3. tail pool
// Of the unselected blocks j of row (h, qb), with p_j = exp(bf16(cm_j) - C):
// C = max bf16(cm_j), T[d] = sum_j p_j * vsum[j][d], L = sum_j p_j * len_j, each sum in
// ascending j with one fused multiply-add per term (an all-selected row gives C = -inf,
// T = 0, L = 0). Selected blocks enter the products with p = 0, which leaves a sum's
// bits unchanged, so T and L run as a dense register-tiled product.

// warp per (h, qb): C (a max, so any order)
__global__ void tail_cmax_kernel(const uint8_t* __restrict__ sel, const __nv_bfloat16* __restrict__ cm, int H,
                                 int nb, float* __restrict__ tC) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)H * nb) return;
  const uint8_t* sr = sel + row * nb;
  const __nv_bfloat16* cr = cm + row * nb;
  float cmax = -INFINITY;
  for (int j = lane; j < nb; j += 32)
    if (!sr[j]) cmax = fmaxf(cmax, __bfloat162float(cr[j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
  if (lane == 0) tC[row] = cmax;
}

// grid (ceil(nb/64), H), block 128: T for 64 query blocks x HD columns (8 x HD/16 per
// thread) and L (threads tx == 0); p (64 x 32) and vsum (32 x HD) staged through shared
// memory per chunk of 32 j
template <int HD>
__global__ void __launch_bounds__(128) tail_pool_kernel(const uint8_t* __restrict__ sel,
                                                        const __nv_bfloat16* __restrict__ cm,
                                                        const __nv_bfloat16* __restrict__ vsum,
                                                        const float* __restrict__ lens,
                                                        const float* __restrict__ tC, int nb,
                                                        float* __restrict__ tT, float* __restrict__ tL) {
  constexpr int QB = 64, JC = 32, ND = HD / 16, QT = 8;
  __shared__ float ps[QB][JC + 1];
  __shared__ float vs[JC][HD];
  __shared__ float ls[JC];
  const int h = blockIdx.y, qb0 = blockIdx.x * QB;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 8 groups of 8 query blocks
  float acc[QT][ND], accl[QT];
#pragma unroll
  for (int i = 0; i < QT; ++i) {
    accl[i] = 0.f;
#pragma unroll
    for (int k = 0; k < ND; ++k) acc[i][k] = 0.f;
  }
  const int64_t hrow = (int64_t)h * nb;
  for (int j0 = 0; j0 < nb; j0 += JC) {
    __syncthreads();
    for (int e = threadIdx.x; e < QB * JC; e += 128) {
      const int r = e / JC, jj = e % JC;
      const int qb = qb0 + r, j = j0 + jj;
      float pv = 0.f;
      if (qb < nb && j < nb) {
        const int64_t idx = (hrow + qb) * nb + j;
        const float c = __ldg(tC + hrow + qb);
        if (!sel[idx] && c > -INFINITY) pv = expf(__bfloat162float(cm[idx]) - c);
      }
      ps[r][jj] = pv;
    }
    for (int e = threadIdx.x; e < JC * HD; e += 128) {
      const int jj = e / HD, d = e % HD, j = j0 + jj;
      vs[jj][d] = j < nb ? __bfloat162float(vsum[(hrow + j) * HD + d]) : 0.f;
    }
    if (threadIdx.x < JC) ls[threadIdx.x] = j0 + threadIdx.x < nb ? lens[j0 + threadIdx.x] : 0.f;
    __syncthreads();
#pragma unroll 2
    for (int jj = 0; jj < JC; ++jj) {
      float pq[QT], vv[ND];
#pragma unroll
      for (int i = 0; i < QT; ++i) pq[i] = ps[ty * QT + i][jj];
#pragma unroll
      for (int k = 0; k < ND; ++k) vv[k] = vs[jj][tx + 16 * k];
#pragma unroll
      for (int i = 0; i < QT; ++i)
#pragma unroll
        for (int k = 0; k < ND; ++k) acc[i][k] = __fmaf_rn(pq[i], vv[k], acc[i][k]);
      if (tx == 0) {
        const float lj = ls[jj];
#pragma unroll
        for (int i = 0; i < QT; ++i) accl[i] = __fmaf_rn(pq[i], lj, accl[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < QT; ++i) {
    const int qb = qb0 + ty * QT + i;
    if (qb >= nb) continue;
#pragma unroll
    for (int k = 0; k < ND; ++k) tT[(hrow + qb) * HD + tx + 16 * k] = acc[i][k];
    if (tx == 0) tL[hrow + qb] = accl[i];
  }
}

// ------------------------------------------------------------ 4. kept lists
// warp per (h, t): number of list entries of video q tile t
__global__ void list_count_kernel(const uint8_t* __restrict__ sel, int H, int nb, int nvt, int qpb,
                                  int* __restrict__ counts) {
  const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)H * nvt) return;
  const int h = (int)(wid / nvt), t = (int)(wid % nvt);
  int cnt = 0;
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    bool u = false;
    if (kb < nb)
      for (int e = 0; e < qpb; ++e) {
        const int qb = t * qpb + e;
        if (qb < nb && sel[((int64_t)h * nb + qb) * nb + kb]) u = true;
      }
    cnt += __popc(__ballot_sync(0xffffffffu, u));
  }
  if (lane == 0) counts[wid] = (cnt + (qpb - 1)) / qpb;  // qpb == kpt: 2 halves per entry for 64-blocks
}

// single block: exclusive scan of counts[n] into offsets[n+1]
__global__ void scan_kernel(const int* __restrict__ counts, int n, int* __restrict__ offsets) {
  __shared__ int part[1024];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int chunk = (n + nt - 1) / nt;
  const int b = tid * chunk, e = min(n, b + chunk);
  int s = 0;
  for (int i = b; i < e; ++i) s += counts[i];
  part[tid] = s;
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int i = 0; i < nt; ++i) {
      int v = part[i];
      part[i] = run;
      run += v;
    }
    offsets[n] = run;
  }
  __syncthreads();
  int run = part[tid];
  for (int i = b; i < e; ++i) {
    offsets[i] = run;
    run += counts[i];
  }
}

// warp per (h, t): write the entries {start0, start1, len0|qmask0<<8, len1|qmask1<<8}
__global__ void list_fill_kernel(const uint8_t* __restrict__ sel, int H, int nb, int nvt, int qpb, int block,
                                 int64_t g, int64_t S, const int* __restrict__ offsets, int4* __restrict__ entries) {
  const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)H * nvt) return;
  const int h = (int)(wid / nvt), t = (int)(wid % nvt);
  int* base = reinterpret_cast<int*>(entries + offsets[wid]);
  int pos0 = 0;
  int total = 0;
  // total union count (for the odd-tail padding)
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    bool u = false;
    if (kb < nb)
      for (int e = 0; e < qpb; ++e) {
        const int qb = t * qpb + e;
        if (qb < nb && sel[((int64_t)h * nb + qb) * nb + kb]) u = true;
      }
    total += __popc(__ballot_sync(0xffffffffu, u));
  }
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    uint32_t qm = 0;
    if (kb < nb)
      for (int e = 0; e < qpb; ++e) {
        const int qb = t * qpb + e;
        if (qb < nb && sel[((int64_t)h * nb + qb) * nb + kb]) qm |= 1u << e;
      }
    const uint32_t bal = __ballot_sync(0xffffffffu, qm != 0);
    if (qm) {
      const int pos = pos0 + __popc(bal & ((1u << lane) - 1u));
      const int64_t start = g + (int64_t)kb * block;
      if (block == 64) {
        const int len = (int)min64(64, S - start);
        const int slot = pos & 1;
        int* ent = base + (pos >> 1) * 4;
        ent[slot] = (int)start;
        ent[2 + slot] = len | (int)(qm << 8);
        if (slot == 0 && pos == total - 1) {  // odd count: empty second half
          ent[1] = (int)start;
          ent[3] = 0;
        }
      } else {  // 128-row blocks: both q halves share the decision
        const int len0 = (int)max64(0, min64(64, S - start));
        const int len1 = (int)max64(0, min64(64, S - start - 64));
        int* ent = base + pos * 4;
        ent[0] = (int)start;
        ent[1] = (int)(start + 64);
        ent[2] = len0 | (3 << 8);
        ent[3] = len1 | (3 << 8);
      }
    }
    pos0 += __popc(bal);
  }
}

// thread per item: strip/dense items first (the heaviest), then video tiles;
// head-major within each group so that the CTAs resident at one time share
// one head's K/V in L2
// Item order: first the PAIRED strip / dense items (pair p = items 2p, 2p+1: two
// consecutive query tiles of one head, both walking every key tile), then the
// unpaired strip tile of each head when the head has an odd number, then the
// video items (head-major). npair_h = pairs per head (0 when pairing is off).
__global__ void items_kernel(int H, int nst, int nvt, int64_t S, int64_t g, int dense_all, int qpb, int nb,
                             int npair_h, const int* __restrict__ offsets, WorkItem* __restrict__ items) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t n_strip = (int64_t)H * nst;
  const int64_t n_items = n_strip + (int64_t)H * nvt;
  if (i == 0) items[n_items].q_start = 0;  // work counter of the persistent flash kernel
  if (i >= n_items) return;
  const int64_t n_paired = 2 * (int64_t)H * npair_h;
  const int n_rest = nst - 2 * npair_h;  // unpaired strip tiles per head
  WorkItem it;
  it.pad0 = it.pad1 = it.pad2 = 0;
  const int kt_all = (int)((S + 127) / 128);
  int strip_h = -1, strip_t = 0;
  if (i < n_paired) {
    const int64_t pr = i >> 1;
    strip_h = (int)(pr / npair_h);
    strip_t = 2 * (int)(pr % npair_h) + (int)(i & 1);
  } else if (i < n_strip) {
    const int64_t r = i - n_paired;
    strip_h = (int)(r / n_rest);
    strip_t = 2 * npair_h + (int)(r % n_rest);
  }
  if (strip_h >= 0) {
    const int t = strip_t;
    it.head = strip_h;
    it.q_start = t * 128;
    const int64_t lim = dense_all ? S : g;
    it.q_rows = (int)min64(128, lim - (int64_t)t * 128);
    it.tail0 = it.tail1 = -1;
    it.list_begin = 0;
    it.list_len = 0;
    it.n_implicit = kt_all;
    it.implicit_end = (int)S;
  } else {
    const int64_t j = i - n_strip;
    const int t = (int)(j % nvt);
    const int h = (int)(j / nvt);
    it.head = h;
    it.q_start = (int)(g + (int64_t)t * 128);
    it.q_rows = (int)min64(128, S - it.q_start);
    it.tail0 = t * qpb;
    it.tail1 = (t * qpb + qpb - 1 < nb) ? t * qpb + qpb - 1 : -1;
    const int64_t w = (int64_t)h * nvt + t;
    it.list_begin = offsets[w];
    it.list_len = offsets[w + 1] - offsets[w];
    it.n_implicit = (int)((g + 127) / 128);
    it.implicit_end = (int)g;
  }
  items[i] = it;
}

// ------------------------------------------------------------ 5. flash kernel
#include "wx_flash.cuh"
#include "wx_flash2.cuh"
#include "wx_flash5.cuh"

// ------------------------------------------------------------- host driver
struct AttnGeom {
  int64_t S, g;
  int H, hd, block, nb, nvt, nst, qpb;
  bool dense;
};

static size_t route_bytes(const AttnGeom& a, int mode) {
  Carve c;
  const size_t hnb = (size_t)a.H * a.nb;
  c.take(hnb * a.hd * 4);           // qc
  c.take(hnb * a.hd * 4);           // kc
  c.take((size_t)a.H * a.hd * 4);   // kvar
  c.take(hnb * 4);                  // thr
  c.take(hnb * a.nb * 2);           // cm
  c.take(hnb * a.nb);               // sel
  if (mode == WX_SPARSE_TOPK) c.take(hnb * a.nb * 4);  // scores
  c.take(hnb * a.hd * 2);           // vsum
  c.take((size_t)a.nb * 4);         // lens
  return c.off;
}

static size_t list_bytes(const AttnGeom& a) {
  Carve c;
  const size_t hnb = (size_t)a.H * a.nb;
  c.take(hnb * a.hd * 4);  // tailT
  c.take(hnb * 4);         // tailL
  c.take(hnb * 4);         // tailC
  c.take((size_t)a.H * a.nvt * 4);            // counts
  c.take(((size_t)a.H * a.nvt + 1) * 4);      // offsets
  c.take((size_t)a.H * a.nvt * (size_t)((a.nb + a.qpb - 1) / a.qpb + 1) * 16);  // entries (worst case)
  c.take(((size_t)a.H * (a.nst + a.nvt) + 1) * sizeof(WorkItem));  // + work counter
  return c.off;
}

static int geom_from(wx_ctx* ctx, int64_t S, int H, int hd, const wx_sparse_spec* spec, AttnGeom& a) {
  a.S = S;
  a.H = H;
  a.hd = hd;
  a.dense = !spec || spec->mode == WX_SPARSE_DENSE;
  if (a.dense) {
    a.g = 0;
    a.block = 128;
    a.nb = 0;
    a.nvt = 0;
    a.qpb = 1;
    a.nst = (int)((S + 127) / 128);
    return WX_OK;
  }
  a.g = spec->g;
  a.block = spec->block;
  if (a.block != 64 && a.block != 128)
    return set_error(ctx, WX_ERR_UNSUPPORTED, "sparse block must be 64 or 128 (got %d)", a.block);
  if (a.g < 0 || a.g >= S) return set_error(ctx, WX_ERR_INVALID, "strip rows g=%lld must be in [0, S)", (long long)a.g);
  a.nb = (int)((S - a.g + a.block - 1) / a.block);
  a.qpb = 128 / a.block;
  a.nvt = (a.nb + a.qpb - 1) / a.qpb;
  a.nst = (int)((a.g + 127) / 128);
  return WX_OK;
}

static int run_routing(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, const AttnGeom& a,
                       const wx_sparse_spec* spec, float scale, uint8_t* base, uint8_t** sel_out,
                       __nv_bfloat16** cm_out, __nv_bfloat16** vsum_out, float** lens_out, float** thr_out,
                       float** scores_out) {
  Carve c;
  const size_t hnb = (size_t)a.H * a.nb;
  float* qc = reinterpret_cast<float*>(base + c.take(hnb * a.hd * 4));
  float* kc = reinterpret_cast<float*>(base + c.take(hnb * a.hd * 4));
  float* kvar = reinterpret_cast<float*>(base + c.take((size_t)a.H * a.hd * 4));
  float* thr = reinterpret_cast<float*>(base + c.take(hnb * 4));
  __nv_bfloat16* cm = reinterpret_cast<__nv_bfloat16*>(base + c.take(hnb * a.nb * 2));
  uint8_t* sel = base + c.take(hnb * a.nb);
  float* scores = nullptr;
  if (spec->mode == WX_SPARSE_TOPK) scores = reinterpret_cast<float*>(base + c.take(hnb * a.nb * 4));
  __nv_bfloat16* vsum = reinterpret_cast<__nv_bfloat16*>(base + c.take(hnb * a.hd * 2));
  float* lens = reinterpret_cast<float*>(base + c.take((size_t)a.nb * 4));
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  ProfScope prof(ctx, kProfRoute);
  block_stats_kernel<<<dim3(a.nb, a.H), a.hd, 0, ctx->stream>>>(Q, K, V, rs, a.S, a.hd, a.g, a.block, a.nb, qc, kc,
                                                                  vsum, lens);
  int st = launch_status(ctx, "block_stats");
  if (st) return st;
  if (spec->mode == WX_SPARSE_SOL) {
    kcenter_kernel<<<a.H, a.hd, 0, ctx->stream>>>(kc, a.nb, a.hd, kvar);
    thr_kernel<<<(unsigned)((hnb + 127) / 128), 128, 0, ctx->stream>>>(qc, kvar, a.H, a.nb, a.hd, scale,
                                                                        spec->tau, thr);
  }
  if (a.hd % 32 != 0) return set_error(ctx, WX_ERR_UNSUPPORTED, "routing needs head_dim %% 32 == 0");
  dim3 sg((a.nb + 63) / 64, (a.nb + 63) / 64, a.H);
  score_kernel<<<sg, 256, 0, ctx->stream>>>(qc, kc, a.nb, a.hd, scale, spec->mode, thr, spec->sink_start,
                                           spec->sink_end, cm, sel, scores);
  st = launch_status(ctx, "score", spec->mode == WX_SPARSE_SOL ? 3 : 1);
  if (st) return st;
  if (spec->mode == WX_SPARSE_TOPK) {
    if (a.nb > 16384) return set_error(ctx, WX_ERR_UNSUPPORTED, "top-k router supports at most 16384 blocks");
    double want = ceil((double)spec->density * (double)a.nb);
    int keep = (int)std::min<double>(want, a.nb - 1);
    if (keep < 0) keep = 0;
    const size_t smem = (size_t)a.nb * 4;
    if (smem > 48 * 1024 && (st = ensure_smem_attr(ctx, (const void*)topk_select_kernel, (int)smem, "topk_select")))
      return st;
    topk_select_kernel<<<dim3(a.nb, a.H), 256, smem, ctx->stream>>>(scores, a.nb, keep, sel);
    st = launch_status(ctx, "topk_select");
    if (st) return st;
  }
  *sel_out = sel;
  *cm_out = cm;
  *vsum_out = vsum;
  *lens_out = lens;
  if (thr_out) *thr_out = thr;
  if (scores_out) *scores_out = scores;
  return WX_OK;
}

// The register split of the paired / duo kernels (setmaxnreg) must fit the register
// file the launch reserves: check the compiled per-thread count once per instantiation.
template <bool DUO, int HD>
static bool flash_pair_regs_ok() {
  static const int ok = [] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, (const void*)flash_attn_pair_kernel<DUO, HD>) == cudaSuccess &&
           fa.numRegs * kA5Threads >= kRegsLow * 128 + kRegsHigh * 256;
  }();
  return ok != 0;
}

// Two routed items per CTA (flash_attn_pair_kernel<true, HD>; WX_ATTN_DUO, read once; 0 =
// routed items in flash_attn2_kernel instead, head_dim 128 only).
static int attn_duo() {
  static int v = [] {
    const char* e = getenv("WX_ATTN_DUO");
    return (e && atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

// Pair strip / dense query tiles that walk the same key tiles (WX_ATTN_PAIRS, read once; 0 = off).
static int attn_pairs() {
  static int v = [] {
    const char* e = getenv("WX_ATTN_PAIRS");
    return (e && atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

bool attn_peer_path_ok() { return attn_duo() && flash_pair_regs_ok<false, 128>() && flash_pair_regs_ok<true, 128>(); }

static int run_flash(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, const AttnGeom& a,
                     const wx_sparse_spec* spec, float scale, const uint8_t* sel, const __nv_bfloat16* cm,
                     const __nv_bfloat16* vsum, const float* lens, uint8_t* base, void* out, int64_t os,
                     const SpPeerOut* po = nullptr) {
  Carve c;
  const size_t hnb = (size_t)a.H * a.nb;
  float* tT = reinterpret_cast<float*>(base + c.take(hnb * a.hd * 4));
  float* tL = reinterpret_cast<float*>(base + c.take(hnb * 4));
  float* tC = reinterpret_cast<float*>(base + c.take(hnb * 4));
  int* counts = reinterpret_cast<int*>(base + c.take((size_t)a.H * a.nvt * 4));
  int* offsets = reinterpret_cast<int*>(base + c.take(((size_t)a.H * a.nvt + 1) * 4));
  const size_t n_entries = (size_t)a.H * a.nvt * (size_t)((a.nb + a.qpb - 1) / a.qpb + 1);
  int4* entries = reinterpret_cast<int4*>(base + c.take(n_entries * 16));
  WorkItem* items =
      reinterpret_cast<WorkItem*>(base + c.take(((size_t)a.H * (a.nst + a.nvt) + 1) * sizeof(WorkItem)));
  const bool tail = !a.dense && spec->tail && cm && vsum && lens;
  const int64_t n_items = (int64_t)a.H * (a.nst + a.nvt);
  // strip / dense query tiles walk every key tile: pair them to share K/V loads
  const int npair_h = attn_pairs() ? a.nst / 2 : 0;
  const int64_t n_pairs = (int64_t)a.H * npair_h;
  int st;
  {
  ProfScope prof(ctx, kProfRoute);
  if (!a.dense) {
    if (tail) {
      tail_cmax_kernel<<<(unsigned)((hnb * 32 + 255) / 256), 256, 0, ctx->stream>>>(sel, cm, a.H, a.nb, tC);
      const dim3 tg((a.nb + 63) / 64, a.H);
      if (a.hd == 64)
        tail_pool_kernel<64><<<tg, 128, 0, ctx->stream>>>(sel, cm, vsum, lens, tC, a.nb, tT, tL);
      else
        tail_pool_kernel<128><<<tg, 128, 0, ctx->stream>>>(sel, cm, vsum, lens, tC, a.nb, tT, tL);
      if ((st = launch_status(ctx, "tail", 2))) return st;
    }
    const int64_t warps = (int64_t)a.H * a.nvt;
    const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
    list_count_kernel<<<blocks, 256, 0, ctx->stream>>>(sel, a.H, a.nb, a.nvt, a.qpb, counts);
    scan_kernel<<<1, 1024, 0, ctx->stream>>>(counts, a.H * a.nvt, offsets);
    list_fill_kernel<<<blocks, 256, 0, ctx->stream>>>(sel, a.H, a.nb, a.nvt, a.qpb, a.block, a.g, a.S, offsets,
                                                      entries);
    if ((st = launch_status(ctx, "list build", 3))) return st;
  }

  items_kernel<<<(unsigned)((n_items + 127) / 128), 128, 0, ctx->stream>>>(a.H, a.nst, a.nvt, a.S, a.g, a.dense,
                                                                             a.qpb, a.nb, npair_h, offsets, items);
  if ((st = launch_status(ctx, "items"))) return st;
  }

  const int64_t cols = (int64_t)a.H * a.hd;
  CUtensorMap tq, tk, tv;
  if ((st = make_tmap_bf16_2d(ctx, &tq, q, (uint64_t)a.S, (uint64_t)cols, (uint64_t)rs, 64, 64))) return st;
  if ((st = make_tmap_bf16_2d(ctx, &tk, k, (uint64_t)a.S, (uint64_t)cols, (uint64_t)rs, 64, 64))) return st;
  if ((st = make_tmap_bf16_2d(ctx, &tv, v, (uint64_t)a.S, (uint64_t)cols, (uint64_t)rs, 64, 64))) return st;
  {
    struct KS {
      const void* fn;
      int bytes;
    };
    const KS ks[] = {{(const void*)flash_attn2_kernel, kA2Smem},
                     {(const void*)flash_attn_pair_kernel<false, 128>, A5Geom<128>::kSmem},
                     {(const void*)flash_attn_pair_kernel<true, 128>, A5Geom<128>::kSmem},
                     {(const void*)flash_attn_pair_kernel<false, 64>, A5Geom<64>::kSmem},
                     {(const void*)flash_attn_pair_kernel<true, 64>, A5Geom<64>::kSmem}};
    for (const KS& k2 : ks)
      if ((st = ensure_smem_attr(ctx, k2.fn, k2.bytes, "flash attention"))) return st;
  }
  AttnParams p{};
  p.items = items;
  p.entries = entries;
  p.tailT = tail ? tT : nullptr;
  p.tailL = tL;
  p.tailC = tC;
  p.nqb = a.nb;
  p.H = a.H;
  p.sl2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = os;
  p.err = ctx->dev_err;
  p.S = a.S;
  p.n_entries = (int64_t)n_entries;
  p.P = po ? po->P : 0;
  if (po) {
    static_assert(kSpMaxPeers == kMaxPeers, "peer table sizes");
    if (!attn_peer_path_ok() || po->P < 1 || po->P > kMaxPeers || po->rows <= 0)
      return set_error(ctx, WX_ERR_UNSUPPORTED, "attention to peer memory needs the paired / duo kernels");
    const int64_t n_rest = n_items - 2 * n_pairs;
    for (int r = 0; r < kMaxPeers; ++r) {
      p.out_peer[r] = r < po->P ? static_cast<__nv_bfloat16*>(po->out_peer[r]) : nullptr;
      p.sig.flags[r] = r < po->P ? po->flags[r] : nullptr;
    }
    p.peer_rows = po->rows;
    p.peer_col = po->col;
    p.sig.counter = po->counter;
    p.sig.total = (int)(n_pairs + (n_rest + 1) / 2);  // CTAs of the paired and the duo launch
    p.sig.P = po->P;
    p.sig.rank = po->rank;
    p.sig.epoch = po->epoch;
  }

  if (n_items > INT32_MAX) return set_error(ctx, WX_ERR_UNSUPPORTED, "too many attention work items");
  ProfScope prof(ctx, kProfAttn);
  const bool hd64 = a.hd == 64;
  // The paired (strip / dense) items are few and long, the routed ones many and short:
  // the routed kernel runs on a side stream so that its CTAs fill the SMs left idle by
  // the last, partial wave of paired CTAs.
  const int64_t n_rest = n_items - 2 * n_pairs;
  const bool duo = attn_duo() && (hd64 ? flash_pair_regs_ok<true, 64>() : flash_pair_regs_ok<true, 128>());
  if (n_rest > 0 && !duo && (hd64 || po))
    return set_error(ctx, WX_ERR_UNSUPPORTED, "%s needs the two-item attention kernel (WX_ATTN_DUO=0 or its register "
                     "split does not fit)", hd64 ? "head_dim 64" : "attention to peer memory");
  const bool side = n_pairs > 0 && n_rest > 0 && duo;
  if (side) {
    if (!ctx->aux) {
      cudaError_t e = cudaStreamCreateWithFlags(&ctx->aux, cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->fork, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->join, cudaEventDisableTiming);
      if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "side stream: %s", cudaGetErrorString(e));
    }
    cudaEventRecord(ctx->fork, ctx->stream);  // after the routing / item kernels
    cudaStreamWaitEvent(ctx->aux, ctx->fork, 0);
  }
  if (n_pairs > 0) {
    const bool regs = hd64 ? flash_pair_regs_ok<false, 64>() : flash_pair_regs_ok<false, 128>();
    if (!regs) return set_error(ctx, WX_ERR_CUDA, "flash_attn_pair: register split does not fit");
    const int np2 = (int)(2 * n_pairs);
    if (hd64)
      flash_attn_pair_kernel<false, 64><<<(unsigned)n_pairs, kA5Threads, A5Geom<64>::kSmem, ctx->stream>>>(
          tq, tk, tv, p, np2);
    else
      flash_attn_pair_kernel<false, 128><<<(unsigned)n_pairs, kA5Threads, A5Geom<128>::kSmem, ctx->stream>>>(
          tq, tk, tv, p, np2);
    if ((st = launch_status(ctx, "flash_attn_pair"))) return st;
  }
  // the remaining (unpaired) items
  p.items = items + 2 * n_pairs;
  if (n_rest == 0) return WX_OK;
  if (duo) {
    // two independent (routed) items per CTA, their exponential phases taking turns
    const unsigned grid = (unsigned)((n_rest + 1) / 2);
    const int nr = (int)n_rest;
    cudaStream_t sm = side ? ctx->aux : ctx->stream;
    if (hd64)
      flash_attn_pair_kernel<true, 64><<<grid, kA5Threads, A5Geom<64>::kSmem, sm>>>(tq, tk, tv, p, nr);
    else
      flash_attn_pair_kernel<true, 128><<<grid, kA5Threads, A5Geom<128>::kSmem, sm>>>(tq, tk, tv, p, nr);
    st = launch_status(ctx, "flash_attn_duo");
    if (side) {  // join: the context stream continues after both kernels
      cudaEventRecord(ctx->join, ctx->aux);
      cudaStreamWaitEvent(ctx->stream, ctx->join, 0);
    }
    return st;
  }
  // fallback for the routed items (head_dim 128): one item per CTA, two CTAs per SM
  flash_attn2_kernel<<<(unsigned)n_rest, kAttnThreads, kA2Smem, ctx->stream>>>(tq, tk, tv, p);
  return launch_status(ctx, "flash_attn2");
}

static int check_attn_args(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S, int H,
                           int hd, const void* out, int64_t os) {
  WX_CHECK_ARG(ctx, ctx && q && k && v && out && S > 0 && H > 0);
  if (hd != 128 && hd != 64)
    return set_error(ctx, WX_ERR_UNSUPPORTED, "attention head_dim must be 128 or 64 (got %d)", hd);
  WX_CHECK_ARG(ctx, rs >= (int64_t)H * hd && os >= (int64_t)H * hd && rs % 8 == 0 && os % 8 == 0);
  WX_CHECK_ARG(ctx, aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out));
  WX_CHECK_ARG(ctx, S < (int64_t)1 << 30);
  return WX_OK;
}

size_t attention_scratch_bytes(int64_t S, int H, int hd, const wx_sparse_spec* spec) {
  AttnGeom a;
  if (geom_from(nullptr, S, H, hd, spec, a)) return 0;
  return (a.dense ? 0 : route_bytes(a, spec->mode)) + list_bytes(a) + (size_t(64) << 10);
}

// routing + flash with caller scratch (used by the block forward)
int attention_with_scratch(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S, int H,
                           int hd, const wx_sparse_spec* spec, float scale, void* out, int64_t os, void* scratch) {
  return attention_with_scratch_peer(ctx, q, k, v, rs, S, H, hd, spec, scale, out, os, scratch, nullptr);
}

int attention_with_scratch_peer(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S,
                                int H, int hd, const wx_sparse_spec* spec, float scale, void* out, int64_t os,
                                void* scratch, const SpPeerOut* po) {
  AttnGeom a;
  int st = geom_from(ctx, S, H, hd, spec, a);
  if (st) return st;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  uint8_t* sel = nullptr;
  __nv_bfloat16 *cm = nullptr, *vsum = nullptr;
  float* lens = nullptr;
  size_t off = 0;
  if (!a.dense) {
    st = run_routing(ctx, q, k, v, rs, a, spec, scale, base, &sel, &cm, &vsum, &lens, nullptr, nullptr);
    if (st) return st;
    off = (route_bytes(a, spec->mode) + 255) & ~size_t(255);
  }
  return run_flash(ctx, q, k, v, rs, a, spec, scale, sel, cm, vsum, lens, base + off, out, os, po);
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_sparse_attention(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride, int64_t S,
                        int H, int head_dim, const wx_sparse_spec* spec, float scale, void* out,
                        int64_t out_stride) {
  int st = check_attn_args(ctx, q, k, v, row_stride, S, H, head_dim, out, out_stride);
  if (st) return st;
  AttnGeom a;
  if ((st = geom_from(ctx, S, H, head_dim, spec, a))) return st;
  void* ws = workspace(ctx, attention_scratch_bytes(S, H, head_dim, spec), &st);
  if (!ws) return st;
  return attention_with_scratch(ctx, q, k, v, row_stride, S, H, head_dim, spec, scale, out, out_stride, ws);
}

static int route_api(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S, int H, int hd,
                     const wx_sparse_spec* spec, float scale, int want_mode, uint8_t* sel, float* thr_or_scores,
                     void* cm, void* vsum, float* lens) {
  WX_CHECK_ARG(ctx, ctx && q && k && v && spec && sel && cm && vsum && lens && S > 0 && H > 0);
  WX_CHECK_ARG(ctx, spec->mode == want_mode);
  if (hd != 128 && hd != 64) return set_error(ctx, WX_ERR_UNSUPPORTED, "routing head_dim must be 128 or 64");
  AttnGeom a;
  int st = geom_from(ctx, S, H, hd, spec, a);
  if (st) return st;
  void* ws = workspace(ctx, route_bytes(a, spec->mode), &st);
  if (!ws) return st;
  uint8_t* dsel;
  __nv_bfloat16 *dcm, *dvs;
  float *dl, *dthr, *dsc;
  st = run_routing(ctx, q, k, v, rs, a, spec, scale, static_cast<uint8_t*>(ws), &dsel, &dcm, &dvs, &dl, &dthr, &dsc);
  if (st) return st;
  const size_t hnb = (size_t)a.H * a.nb;
  cudaStream_t s = ctx->stream;
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(sel, dsel, hnb * a.nb, cudaMemcpyDeviceToDevice, s));
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(cm, dcm, hnb * a.nb * 2, cudaMemcpyDeviceToDevice, s));
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(vsum, dvs, hnb * a.hd * 2, cudaMemcpyDeviceToDevice, s));
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(lens, dl, (size_t)a.nb * 4, cudaMemcpyDeviceToDevice, s));
  if (thr_or_scores) {
    const float* src = want_mode == WX_SPARSE_SOL ? dthr : dsc;
    const size_t n = want_mode == WX_SPARSE_SOL ? hnb : hnb * a.nb;
    WX_CUDA_TRY(ctx, cudaMemcpyAsync(thr_or_scores, src, n * 4, cudaMemcpyDeviceToDevice, s));
  }
  return WX_OK;
}

int wx_sol_route(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride, int64_t S, int H,
                 int head_dim, const wx_sparse_spec* spec, float scale, uint8_t* sel, float* thr, void* cm,
                 void* vsum, float* lens) {
  return route_api(ctx, q, k, v, row_stride, S, H, head_dim, spec, scale, WX_SPARSE_SOL, sel, thr, cm, vsum, lens);
}

int wx_topk_route(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride, int64_t S, int H,
                  int head_dim, const wx_sparse_spec* spec, float scale, uint8_t* sel, float* scores, void* cm,
                  void* vsum, float* lens) {
  return route_api(ctx, q, k, v, row_stride, S, H, head_dim, spec, scale, WX_SPARSE_TOPK, sel, scores, cm, vsum,
                   lens);
}

int wx_attention_from_sel(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride, int64_t S,
                          int H, int head_dim, const wx_sparse_spec* spec, float scale, const uint8_t* sel,
                          const void* cm, const void* vsum, const float* lens, void* out, int64_t out_stride) {
  int st = check_attn_args(ctx, q, k, v, row_stride, S, H, head_dim, out, out_stride);
  if (st) return st;
  WX_CHECK_ARG(ctx, spec && spec->mode != WX_SPARSE_DENSE && sel);
  WX_CHECK_ARG(ctx, !spec->tail || (cm && vsum && lens));
  AttnGeom a;
  if ((st = geom_from(ctx, S, H, head_dim, spec, a))) return st;
  void* ws = workspace(ctx, list_bytes(a) + 1024, &st);
  if (!ws) return st;
  return run_flash(ctx, q, k, v, row_stride, a, spec, scale, sel, static_cast<const __nv_bfloat16*>(cm),
                   static_cast<const __nv_bfloat16*>(vsum), lens, static_cast<uint8_t*>(ws), out, out_stride);
}

}  // extern "C"
