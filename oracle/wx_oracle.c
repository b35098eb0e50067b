/*
 * wx_oracle.c — CPU restatement of the reference's video-DiT hot path.
 * TEST INFRASTRUCTURE ONLY (see wx_oracle.h for the parity status).
 *
 * Built with -ffp-contract=off so that every fp32 multiply/add rounds where
 * the C source says it does; the routing functions use explicit fmaf() where
 * their fixed reduction order asks for a fused multiply-add.
 */
#include "wx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int wxo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* OpenMP threads of every later oracle call, whatever OMP_NUM_THREADS says (a launcher such
 * as torchrun sets it to 1); n <= 0 selects every processor the runtime reports */
int wxo_set_num_threads(int n) {
#ifdef _OPENMP
  if (n <= 0) n = omp_get_num_procs();
  omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* ------------------------------------------------------------------ bf16 */
float wxo_bf2f(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t wxo_f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);                                            /* round to nearest even */
  return (uint16_t)(u >> 16);
}

static inline float bf(uint16_t h) { return wxo_bf2f(h); }
static inline float rbf(float f) { return wxo_bf2f(wxo_f2bf(f)); }

void wxo_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = wxo_f2bf(in[i]);
}

void wxo_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = wxo_bf2f(in[i]);
}

/* ------------------------------------------------------------------- RNG */
static inline uint64_t splitmix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline double normal_at(uint64_t key, int64_t i) {
  uint64_t r = splitmix(key ^ splitmix((uint64_t)i));
  double u1 = ((double)((r >> 40) + 1)) * (1.0 / 16777216.0);       /* (0, 1] */
  double u2 = ((double)((r >> 16) & 0xffffffull)) * (1.0 / 16777216.0); /* [0, 1) */
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static inline uint64_t rng_key(uint64_t seed, uint64_t stream) {
  return splitmix(seed * 0xD1B54A32D192ED03ull ^ splitmix(stream + 0x632BE59BD9B4E019ull));
}

void wxo_fill_normal_f32(float* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std) {
  uint64_t key = rng_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = (float)(mean + std * normal_at(key, i));
}

void wxo_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std) {
  uint64_t key = rng_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = wxo_f2bf((float)(mean + std * normal_at(key, i)));
}

/* ---------------------------------------------------------- quantization */
static int quant_geometry_ok(int64_t k, int group, int bits) {
  if (bits < 2 || bits > 8) return 0;
  if (group <= 0 || k <= 0 || k % group) return 0;
  if ((k * bits) % 32) return 0;
  return 1;
}

int wxo_quantize_affine(const float* w, int64_t n, int64_t k, int group, int bits,
                        uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if (!quant_geometry_ok(k, group, bits)) return -1;
  const int64_t words = k * bits / 32;
  const int64_t groups = k / group;
  const int nbins = (1 << bits) - 1;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    uint32_t* row = wq + r * words;
    memset(row, 0, (size_t)words * 4);
    for (int64_t gi = 0; gi < groups; ++gi) {
      const float* src = w + r * k + gi * group;
      float mn = src[0], mx = src[0];
      for (int j = 1; j < group; ++j) {
        if (src[j] < mn) mn = src[j];
        if (src[j] > mx) mx = src[j];
      }
      float sc = (mx - mn) / (float)nbins;
      if (sc < 1e-7f) sc = 1e-7f;
      uint16_t sb = wxo_f2bf(sc), bb = wxo_f2bf(mn);
      scales[r * groups + gi] = sb;
      biases[r * groups + gi] = bb;
      float s = bf(sb), b = bf(bb);
      for (int j = 0; j < group; ++j) {
        float qf = rintf((src[j] - b) / s);
        int q = qf < 0.f ? 0 : (qf > (float)nbins ? nbins : (int)qf);
        int64_t bit = (gi * group + j) * (int64_t)bits;
        int64_t wi = bit >> 5;
        int off = (int)(bit & 31);
        row[wi] |= ((uint32_t)q) << off;
        if (off + bits > 32) row[wi + 1] |= ((uint32_t)q) >> (32 - off);
      }
    }
  }
  return 0;
}

static inline int unpack_q(const uint32_t* row, int64_t i, int bits) {
  int64_t bit = i * (int64_t)bits;
  int64_t wi = bit >> 5;
  int off = (int)(bit & 31);
  uint32_t v = row[wi] >> off;
  if (off + bits > 32) v |= row[wi + 1] << (32 - off);
  return (int)(v & ((1u << bits) - 1u));
}

int wxo_dequantize_affine(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                          int64_t n, int64_t k, int group, int bits, uint16_t* w_out) {
  if (!quant_geometry_ok(k, group, bits)) return -1;
  const int64_t words = k * bits / 32;
  const int64_t groups = k / group;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    const uint32_t* row = wq + r * words;
    for (int64_t i = 0; i < k; ++i) {
      float s = bf(scales[r * groups + i / group]);
      float b = bf(biases[r * groups + i / group]);
      float q = (float)unpack_q(row, i, bits);
      w_out[r * k + i] = wxo_f2bf(q * s + b); /* q*s is exact in fp32 for bits <= 8 */
    }
  }
  return 0;
}

/* --------------------------------------------------------------- qlinear */
static inline float gelu_tanh(float x) {
  const float c = 0.7978845608028654f; /* sqrt(2/pi) */
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

/* t[r][c] = sum over i = 0, 1, ..., k-1 of (double)xf[r][i] * (double)wf[c][i], in that
 * order, for a 4 x 4 block of outputs at once: the sixteen accumulators are independent,
 * so the adds of one output do not wait on one another's latency, and every output still
 * takes exactly the sequence acc = acc + x*w of the one-output loop. Rows/columns past the
 * edge repeat the last valid one and are not stored. */
__attribute__((target_clones("avx2", "default"))) static void dot_block4(const float* xf, int64_t m, const float* wf, int64_t n, int64_t k, int64_t r0, int64_t c0,
                       double* out /* [4][4] */) {
  const float* xr[4];
  const float* wr[4];
  for (int j = 0; j < 4; ++j) {
    const int64_t r = r0 + j < m ? r0 + j : m - 1;
    const int64_t c = c0 + j < n ? c0 + j : n - 1;
    xr[j] = xf + r * k;
    wr[j] = wf + c * k;
  }
  double a00 = 0, a01 = 0, a02 = 0, a03 = 0, a10 = 0, a11 = 0, a12 = 0, a13 = 0;
  double a20 = 0, a21 = 0, a22 = 0, a23 = 0, a30 = 0, a31 = 0, a32 = 0, a33 = 0;
  for (int64_t i = 0; i < k; ++i) {
    const double x0 = xr[0][i], x1 = xr[1][i], x2 = xr[2][i], x3 = xr[3][i];
    const double w0 = wr[0][i], w1 = wr[1][i], w2 = wr[2][i], w3 = wr[3][i];
    a00 += x0 * w0; a01 += x0 * w1; a02 += x0 * w2; a03 += x0 * w3;
    a10 += x1 * w0; a11 += x1 * w1; a12 += x1 * w2; a13 += x1 * w3;
    a20 += x2 * w0; a21 += x2 * w1; a22 += x2 * w2; a23 += x2 * w3;
    a30 += x3 * w0; a31 += x3 * w1; a32 += x3 * w2; a33 += x3 * w3;
  }
  out[0] = a00; out[1] = a01; out[2] = a02; out[3] = a03;
  out[4] = a10; out[5] = a11; out[6] = a12; out[7] = a13;
  out[8] = a20; out[9] = a21; out[10] = a22; out[11] = a23;
  out[12] = a30; out[13] = a31; out[14] = a32; out[15] = a33;
}

int wxo_qlinear(const uint16_t* x, int64_t m, int64_t k,
                const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                int64_t n, int group, int bits, const uint16_t* bias, int epilogue,
                const uint16_t* gate, const uint16_t* resid, const uint32_t* rowmap,
                uint16_t* y, uint16_t* y_raw) {
  if (!quant_geometry_ok(k, group, bits) || m < 0 || n <= 0) return -1;
  if (epilogue == WXO_EPI_SWIGLU && (n & 1)) return -1;
  if (epilogue == WXO_EPI_GATE_RESID && (!gate || !resid)) return -1;
  if (m == 0) return 0;
  uint16_t* wd = (uint16_t*)malloc((size_t)n * k * 2);
  float* wf = (float*)malloc((size_t)n * k * 4);
  float* xf = (float*)malloc((size_t)m * k * 4);
  float* t = (float*)malloc((size_t)m * n * 4);
  if (!wd || !wf || !xf || !t) { free(wd); free(wf); free(xf); free(t); return -2; }
  wxo_dequantize_affine(wq, scales, biases, n, k, group, bits, wd);
  wxo_bf16_to_f32(wd, wf, n * k);
  free(wd);
  wxo_bf16_to_f32(x, xf, m * k);
  /* t = bf16(acc), then bf16(t + bias): 32 x 32 output tiles per task, 4 x 4 blocks inside */
  const int64_t mt = (m + 31) / 32, nt = (n + 31) / 32;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t tile = 0; tile < mt * nt; ++tile) {
    const int64_t rt = (tile / nt) * 32, ct = (tile % nt) * 32;
    double blk[16];
    for (int64_t r0 = rt; r0 < rt + 32 && r0 < m; r0 += 4)
      for (int64_t c0 = ct; c0 < ct + 32 && c0 < n; c0 += 4) {
        dot_block4(xf, m, wf, n, k, r0, c0, blk);
        for (int a = 0; a < 4 && r0 + a < m; ++a)
          for (int b = 0; b < 4 && c0 + b < n; ++b) {
            float tv = rbf((float)blk[a * 4 + b]);
            if (bias) tv = rbf(tv + bf(bias[c0 + b]));
            t[(r0 + a) * n + c0 + b] = tv;
          }
      }
  }
  free(wf);
  free(xf);
  const int64_t F = n / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const float* tr = t + r * n;
    const uint32_t mr = rowmap ? rowmap[r] : 0u;
    if (epilogue == WXO_EPI_SWIGLU) {
      for (int64_t j = 0; j < F; ++j) {
        float gt = tr[j], up = tr[F + j];
        float silu = gt / (1.0f + expf(-gt));
        y[r * F + j] = wxo_f2bf(silu * up);
      }
    } else {
      for (int64_t c = 0; c < n; ++c) {
        float o;
        if (epilogue == WXO_EPI_GELU) o = gelu_tanh(tr[c]);
        else if (epilogue == WXO_EPI_GATE_RESID) o = bf(resid[r * n + c]) + tr[c] * bf(gate[(int64_t)mr * n + c]);
        else o = tr[c];
        y[r * n + c] = wxo_f2bf(o);
        if (y_raw) y_raw[r * n + c] = wxo_f2bf(tr[c]);
      }
    }
  }
  free(t);
  return 0;
}

/* ------------------------------------------------------- row kernels K3-5 */
int wxo_qk_norm_rope(const uint16_t* x, int64_t x_stride, int64_t S, int H, int hd,
                     const uint16_t* w, const uint16_t* cos_t, const uint16_t* sin_t,
                     int rot, float eps, uint16_t* out, int64_t out_stride) {
  if (rot < 0 || rot > hd || (rot & 1)) return -1;
  const int rh = rot / 2;
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < S * H; ++row) {
    const int64_t s = row / H;
    const int h = (int)(row % H);
    const uint16_t* xr = x + s * x_stride + (int64_t)h * hd;
    uint16_t* orow = out + s * out_stride + (int64_t)h * hd;
    float nv[512];
    float sum = 0.f;
    for (int j = 0; j < hd; ++j) {
      float v = bf(xr[j]);
      sum += v * v;
    }
    const float rstd = 1.0f / sqrtf(sum / (float)hd + eps);
    for (int j = 0; j < hd; ++j) nv[j] = rbf(bf(xr[j]) * rstd * bf(w[j]));
    for (int j = 0; j < hd; ++j) {
      float o;
      if (j < rh) {
        float c = bf(cos_t[s * rh + j]), sn = bf(sin_t[s * rh + j]);
        o = nv[j] * c - nv[j + rh] * sn;
      } else if (j < rot) {
        float c = bf(cos_t[s * rh + j - rh]), sn = bf(sin_t[s * rh + j - rh]);
        o = nv[j] * c + nv[j - rh] * sn;
      } else {
        o = nv[j];
      }
      orow[j] = wxo_f2bf(o);
    }
  }
  return 0;
}

int wxo_norm_modscale(const uint16_t* x, int64_t S, int64_t hidden, const uint16_t* w,
                      const uint16_t* shift, const uint16_t* scale, const uint32_t* rowmap,
                      float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < S; ++r) {
    const uint16_t* xr = x + r * hidden;
    const int64_t mr = rowmap ? (int64_t)rowmap[r] : 0;
    float sum = 0.f;
    for (int64_t j = 0; j < hidden; ++j) {
      float v = bf(xr[j]);
      sum += v * v;
    }
    const float rstd = 1.0f / sqrtf(sum / (float)hidden + eps);
    for (int64_t j = 0; j < hidden; ++j) {
      float nv = rbf(bf(xr[j]) * rstd * bf(w[j]));
      float o = nv * (bf(scale[mr * hidden + j]) + 1.0f) + bf(shift[mr * hidden + j]);
      out[r * hidden + j] = wxo_f2bf(o);
    }
  }
  return 0;
}

int wxo_mod_gate(const uint16_t* x, const uint16_t* other, const uint16_t* gate,
                 const uint32_t* rowmap, int64_t S, int64_t hidden, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < S; ++r) {
    const int64_t mr = rowmap ? (int64_t)rowmap[r] : 0;
    for (int64_t j = 0; j < hidden; ++j)
      out[r * hidden + j] = wxo_f2bf(bf(x[r * hidden + j]) + bf(other[r * hidden + j]) * bf(gate[mr * hidden + j]));
  }
  return 0;
}

/* --------------------------------------------------------------- routing */
/* block means / sums over the video segment in a fixed sequential order */
static void block_stats(const uint16_t* src, int64_t row_stride, int64_t S, int H, int hd, int64_t g,
                        int block, int nb, int want_mean, float* outp, const float* lens) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < H; ++h)
    for (int b = 0; b < nb; ++b) {
      for (int d = 0; d < hd; ++d) {
        float acc = 0.f;
        const int64_t r0 = g + (int64_t)b * block;
        for (int r = 0; r < block; ++r) {
          int64_t s = r0 + r;
          if (s >= S) break;
          acc += bf(src[s * row_stride + (int64_t)h * hd + d]);
        }
        outp[((int64_t)h * nb + b) * hd + d] = want_mean ? acc / lens[b] : acc;
      }
    }
}

/* acc[t] = fma-chain over d = 0, 1, ... of qr[d] * kr[t*hd + d] for the next (up to) four
 * key blocks: four independent chains, each in the one-block order */
static inline void score_chains4(const float* qr, const float* kr, int avail, int hd, float* acc) {
  const float* k0 = kr;
  const float* k1 = avail > 1 ? kr + hd : kr;
  const float* k2 = avail > 2 ? kr + 2 * hd : kr;
  const float* k3 = avail > 3 ? kr + 3 * hd : kr;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int d = 0; d < hd; ++d) {
    a0 = fmaf(qr[d], k0[d], a0);
    a1 = fmaf(qr[d], k1[d], a1);
    a2 = fmaf(qr[d], k2[d], a2);
    a3 = fmaf(qr[d], k3[d], a3);
  }
  acc[0] = a0;
  acc[1] = a1;
  acc[2] = a2;
  acc[3] = a3;
}

static int route_common(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                        int64_t S, int H, int hd, int64_t g, int block, int* nb_out,
                        float** qc, float** kc, uint16_t* vsum, float* lens) {
  if (S <= g || block <= 0 || hd <= 0 || H <= 0) return -1;
  const int64_t L = S - g;
  const int nb = (int)((L + block - 1) / block);
  *nb_out = nb;
  for (int b = 0; b < nb; ++b) {
    int64_t len = L - (int64_t)b * block;
    lens[b] = (float)(len < block ? len : block);
  }
  *qc = (float*)malloc((size_t)H * nb * hd * 4);
  *kc = (float*)malloc((size_t)H * nb * hd * 4);
  float* vs = (float*)malloc((size_t)H * nb * hd * 4);
  if (!*qc || !*kc || !vs) { free(*qc); free(*kc); free(vs); return -2; }
  block_stats(q, row_stride, S, H, hd, g, block, nb, 1, *qc, lens);
  block_stats(k, row_stride, S, H, hd, g, block, nb, 1, *kc, lens);
  block_stats(v, row_stride, S, H, hd, g, block, nb, 0, vs, lens);
  if (vsum) wxo_f32_to_bf16(vs, vsum, (int64_t)H * nb * hd);
  free(vs);
  return 0;
}

int wxo_sol_route(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                  int64_t S, int H, int hd, int64_t g, int block, float scale, float tau,
                  int sink_start, int sink_end,
                  uint8_t* sel, float* thr, uint16_t* cm, uint16_t* vsum, float* lens) {
  int nb;
  float *qc = NULL, *kc = NULL;
  int rc = route_common(q, k, v, row_stride, S, H, hd, g, block, &nb, &qc, &kc, vsum, lens);
  if (rc) return rc;
  float* kvar = (float*)malloc((size_t)H * hd * 4);
  /* centre the key centroids: kcc = kc - mean_b(kc); kcVar = mean_b(kcc^2) */
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < H; ++h)
    for (int d = 0; d < hd; ++d) {
      float acc = 0.f;
      for (int b = 0; b < nb; ++b) acc += kc[((int64_t)h * nb + b) * hd + d];
      const float mean = acc / (float)nb;
      float vacc = 0.f;
      for (int b = 0; b < nb; ++b) {
        float c = kc[((int64_t)h * nb + b) * hd + d] - mean;
        kc[((int64_t)h * nb + b) * hd + d] = c;
        vacc += c * c;
      }
      kvar[(int64_t)h * hd + d] = vacc / (float)nb;
    }
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < H; ++h)
    for (int i = 0; i < nb; ++i) {
      const float* qr = qc + ((int64_t)h * nb + i) * hd;
      float var = 0.f;
      for (int d = 0; d < hd; ++d) var += (qr[d] * qr[d]) * kvar[(int64_t)h * hd + d];
      const float th = tau * sqrtf(var * (scale * scale) + 1e-6f);
      thr[(int64_t)h * nb + i] = th;
      float accs[4];
      for (int j = 0; j < nb; ++j) {
        if ((j & 3) == 0) score_chains4(qr, kc + ((int64_t)h * nb + j) * hd, nb - j, hd, accs);
        const float acc = accs[j & 3];
        uint16_t c = wxo_f2bf(acc * scale);
        const int64_t idx = ((int64_t)h * nb + i) * nb + j;
        cm[idx] = c;
        int s = bf(c) > th;
        if (abs(i - j) <= 1) s = 1;
        if (j >= sink_start && j < sink_end) s = 1;
        sel[idx] = (uint8_t)s;
      }
    }
  free(kvar);
  free(qc);
  free(kc);
  return 0;
}

typedef struct {
  float s;
  int j;
} scored_idx;

static int cmp_scored_desc(const void* a, const void* b) {
  const scored_idx* x = (const scored_idx*)a;
  const scored_idx* y = (const scored_idx*)b;
  if (x->s != y->s) return x->s > y->s ? -1 : 1;
  return x->j < y->j ? -1 : (x->j > y->j);
}

int wxo_topk_route(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                   int64_t S, int H, int hd, int64_t g, int block, float scale, float density,
                   uint8_t* sel, float* scores, uint16_t* cm, uint16_t* vsum, float* lens) {
  int nb;
  float *qc = NULL, *kc = NULL;
  int rc = route_common(q, k, v, row_stride, S, H, hd, g, block, &nb, &qc, &kc, vsum, lens);
  if (rc) return rc;
  int keep = (int)ceil((double)density * (double)nb);
  if (keep > nb - 1) keep = nb - 1;
  if (keep < 0) keep = 0;
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < H; ++h)
    for (int i = 0; i < nb; ++i) {
      const float* qr = qc + ((int64_t)h * nb + i) * hd;
      float* sr = scores + ((int64_t)h * nb + i) * nb;
      float accs[4];
      for (int j = 0; j < nb; ++j) {
        if ((j & 3) == 0) score_chains4(qr, kc + ((int64_t)h * nb + j) * hd, nb - j, hd, accs);
        const float acc = accs[j & 3];
        sr[j] = acc * scale;
        cm[((int64_t)h * nb + i) * nb + j] = wxo_f2bf(sr[j]);
      }
      uint8_t* selr = sel + ((int64_t)h * nb + i) * nb;
      /* order the off-diagonal blocks: higher score first, lower index on ties */
      scored_idx* ord = (scored_idx*)malloc((size_t)nb * sizeof(scored_idx));
      int n = 0;
      for (int j = 0; j < nb; ++j) {
        selr[j] = (uint8_t)(j == i);
        if (j != i) {
          ord[n].s = sr[j];
          ord[n].j = j;
          ++n;
        }
      }
      qsort(ord, (size_t)n, sizeof(scored_idx), cmp_scored_desc);
      for (int t = 0; t < keep && t < n; ++t) selr[ord[t].j] = 1;
      free(ord);
    }
  free(qc);
  free(kc);
  return 0;
}

/* ------------------------------------------------------------- attention */
/* Online softmax of up to ATT_G query rows that see the same keys in the same order
 * (strip rows, or the rows of one video query block). Every row takes exactly the
 * one-row sequence of operations: s = sum_d q[d]*k[d] in ascending d (fp32), s *= scale,
 * m2 = max(m, s), a = exp(m - m2), p = exp(s - m2), acc = acc*a + p*v, l = l*a + p.
 * The rows are only interleaved (independent chains), which changes no result. */
#define ATT_G 8
typedef struct {
  float m[ATT_G], l[ATT_G];
  float acc[ATT_G][256];
} soft_group;

__attribute__((target_clones("avx2", "default"))) static void feed_rows_g(soft_group* st, const float (*qv)[256], const uint16_t* k, const uint16_t* v,
                        int64_t row_stride, int h, int hd, int64_t r0, int64_t r1, float scale) {
  float kf[256], vf[256];
  for (int64_t r = r0; r < r1; ++r) {
    const uint16_t* kr = k + r * row_stride + (int64_t)h * hd;
    const uint16_t* vr = v + r * row_stride + (int64_t)h * hd;
    for (int d = 0; d < hd; ++d) {
      kf[d] = bf(kr[d]);
      vf[d] = bf(vr[d]);
    }
    float s[ATT_G];
    for (int j = 0; j < ATT_G; ++j) s[j] = 0.f;
    for (int d = 0; d < hd; ++d)
      for (int j = 0; j < ATT_G; ++j) s[j] += qv[j][d] * kf[d];
    for (int j = 0; j < ATT_G; ++j) {
      const float sj = s[j] * scale;
      const float m2 = sj > st->m[j] ? sj : st->m[j];
      const float a = expf(st->m[j] - m2);
      const float p = expf(sj - m2);
      float* acc = st->acc[j];
      for (int d = 0; d < hd; ++d) acc[d] = acc[d] * a + p * vf[d];
      st->l[j] = st->l[j] * a + p;
      st->m[j] = m2;
    }
  }
}

/* the SOL tail term of one unselected block for every row of the group */
static void feed_tail_g(soft_group* st, float sc, float len, const uint16_t* vs, int hd) {
  for (int j = 0; j < ATT_G; ++j) {
    const float m2 = sc > st->m[j] ? sc : st->m[j];
    const float a = expf(st->m[j] - m2);
    const float p = expf(sc - m2);
    float* acc = st->acc[j];
    if (len > 0.f) {
      for (int d = 0; d < hd; ++d) acc[d] = acc[d] * a + p * bf(vs[d]);
      st->l[j] = st->l[j] * a + p * len;
    } else {
      for (int d = 0; d < hd; ++d) acc[d] *= a;
      st->l[j] *= a;
    }
    st->m[j] = m2;
  }
}

int wxo_sparse_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                         int64_t S, int H, int hd, int64_t g, int block, float scale,
                         const uint8_t* sel, const uint16_t* cm, const uint16_t* vsum,
                         const float* lens, int tail, uint16_t* out, int64_t out_stride) {
  return wxo_sparse_attention_rows(q, k, v, row_stride, S, H, hd, g, block, scale, sel, cm, vsum, lens, tail,
                                   0, S, out, out_stride);
}

int wxo_sparse_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                              int64_t S, int H, int hd, int64_t g, int block, float scale,
                              const uint8_t* sel, const uint16_t* cm, const uint16_t* vsum,
                              const float* lens, int tail, int64_t row0, int64_t row1,
                              uint16_t* out, int64_t out_stride) {
  if (hd > 256 || S <= 0 || row0 < 0 || row1 > S || row0 > row1) return -1;
  if (sel && (S <= g || block <= 0)) return -1;
  const int64_t L = S - g;
  const int nb = sel ? (int)((L + block - 1) / block) : 0;
  /* groups of <= ATT_G consecutive rows with the same keys: strip rows (all of S), or
   * the rows of one video query block */
  int64_t ngroups = 0;
  int64_t* gstart = (int64_t*)malloc((size_t)(row1 - row0 + 1) * sizeof(int64_t));
  if (!gstart) return -2;
  for (int64_t s = row0; s < row1;) {
    int64_t end;
    if (!sel) end = row1;
    else if (s < g) end = g;
    else end = g + ((s - g) / block + 1) * block;
    if (end > row1) end = row1;
    if (end > s + ATT_G) end = s + ATT_G;
    gstart[ngroups++] = s;
    s = end;
  }
  gstart[ngroups] = row1;
#pragma omp parallel for collapse(2) schedule(dynamic, 2)
  for (int h = 0; h < H; ++h)
    for (int64_t gi = 0; gi < ngroups; ++gi) {
      const int64_t s0 = gstart[gi], s1 = gstart[gi + 1];
      soft_group* st = (soft_group*)malloc(sizeof(soft_group));
      float(*qv)[256] = (float(*)[256])malloc(sizeof(float) * ATT_G * 256);
      for (int j = 0; j < ATT_G; ++j) {
        const int64_t s = s0 + j < s1 ? s0 + j : s1 - 1; /* padding rows repeat the last row */
        st->m[j] = -INFINITY;
        st->l[j] = 0.f;
        for (int d = 0; d < hd; ++d) st->acc[j][d] = 0.f;
        for (int d = 0; d < hd; ++d) qv[j][d] = bf(q[s * row_stride + (int64_t)h * hd + d]);
      }
      if (!sel || s0 < g) {
        feed_rows_g(st, (const float(*)[256])qv, k, v, row_stride, h, hd, 0, S, scale);
      } else {
        feed_rows_g(st, (const float(*)[256])qv, k, v, row_stride, h, hd, 0, g, scale);
        const int qb = (int)((s0 - g) / block);
        for (int j = 0; j < nb; ++j) {
          const int64_t idx = ((int64_t)h * nb + qb) * nb + j;
          if (sel[idx]) {
            int64_t r0 = g + (int64_t)j * block, r1 = r0 + block;
            if (r1 > S) r1 = S;
            feed_rows_g(st, (const float(*)[256])qv, k, v, row_stride, h, hd, r0, r1, scale);
          } else if (tail) {
            feed_tail_g(st, bf(cm[idx]), lens[j], vsum + ((int64_t)h * nb + j) * hd, hd);
          }
        }
      }
      for (int64_t s = s0; s < s1; ++s) {
        const int j = (int)(s - s0);
        const float inv = 1.0f / st->l[j];
        uint16_t* orow = out + s * out_stride + (int64_t)h * hd;
        for (int d = 0; d < hd; ++d) orow[d] = wxo_f2bf(st->acc[j][d] * inv);
      }
      free(st);
      free(qv);
    }
  free(gstart);
  return 0;
}

/* ----------------------------------------------------------- fp32 dense */
int wxo_dense_f32(const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                  const float* b, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      double acc = b ? (double)b[c] : 0.0;
      for (int64_t i = 0; i < k; ++i) acc += (double)x[r * k + i] * (double)w[i * n + c];
      y[r * n + c] = (float)acc;
    }
  return 0;
}
