/*
 * wx_oracle.h — CPU restatement of the reference's video-DiT denoising hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * product in wuxianhuabu_b200/: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it. The product path never
 * links or calls it.
 *
 * Parity status: PARTLY UNPINNED. The reference (Swift + MLX + Metal) cannot be
 * built or run here and ships no golden vectors for this path. Pinned:
 *   - the affine dequant definition w = q*scale + bias in fp32, rounded to bf16
 *     (model/minimax h3/H3Common.swift:379-401), and the packed-word bit layout
 *     for 4-bit words that the same function decodes (:389-394);
 *   - the PAB schedule examples written in the reference's comments
 *     (model/2网络算子/网络算子-注意力跨步缓存-通用.swift:68-69, 106-110);
 *   - the SOL self-test tolerances and geometries (网络算子-稀疏注意力-SOL通用.swift:683-915);
 *   - the fused-kernel self-test tolerances (网络算子-融合-RMSNormRoPE-通用.swift:349-518).
 * Unpinned: the 6-bit packing layout inside the uint32 words (assumed to be the
 * same little-endian bit stream as the 4-bit case), the MLX affine quantizer's
 * rounding rule (this file's quantizer only manufactures synthetic weights),
 * and MLX's reduction orders (this file fixes its own, which the GPU copies for
 * the bit-exact routing decisions).
 *
 * All bf16 values are carried as uint16_t bit patterns.
 */
#ifndef WX_ORACLE_H
#define WX_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* epilogue codes shared with the CUDA library (include/wx_api.h) */
#define WXO_EPI_NONE 0
#define WXO_EPI_GELU 1
#define WXO_EPI_GATE_RESID 2
#define WXO_EPI_SWIGLU 3

float wxo_bf2f(uint16_t h);
uint16_t wxo_f2bf(float f);
void wxo_f32_to_bf16(const float* in, uint16_t* out, int64_t n);
void wxo_bf16_to_f32(const uint16_t* in, float* out, int64_t n);

/* Counter-based normal generator (splitmix64 + Box-Muller). Element i of
 * (seed, stream) is a pure function of (seed, stream, i). */
void wxo_fill_normal_f32(float* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std);
void wxo_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std);

/* Affine group quantizer used to manufacture synthetic weights:
 * per group of `group` values along K: scale = bf16(max((max-min)/(2^bits-1), 1e-7)),
 * bias = bf16(min), q = clamp(rint((w - bias)/scale), 0, 2^bits-1).
 * Packing: value i of a row sits at bits [i*bits, i*bits+bits) of the row's
 * little-endian bit stream of uint32 words (row = K*bits/32 words). */
int wxo_quantize_affine(const float* w, int64_t n, int64_t k, int group, int bits,
                        uint32_t* wq, uint16_t* scales, uint16_t* biases);
/* w_out[n][k] = bf16(float(q) * scale + bias) (H3Common.swift:379-401) */
int wxo_dequantize_affine(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                          int64_t n, int64_t k, int group, int bits, uint16_t* w_out);

/* MfLinear.forward, quantized branch (H3Common.swift:341-377) plus the fused
 * epilogues the CUDA GEMM applies:
 *   t   = bf16(acc)            (quantizedMM output, acc = fp64 dot of x and deq(W))
 *   t   = bf16(t + bias)       (when bias != NULL, H3Common.swift:366-368)
 *   NONE:       y = t
 *   GELU:       y = bf16(gelu_tanh(t))           (算子-激活.swift:19-21)
 *   GATE_RESID: y = bf16(resid + t * gate[map[m]]) (fused mod_gate, fused:179-196);
 *               y_raw (optional) = t
 *   SWIGLU:     n = 2F; y[m][j] = bf16(silu(t[j]) * t[F+j]) (H3Transformer.swift:620-630)
 */
int wxo_qlinear(const uint16_t* x, int64_t m, int64_t k,
                const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                int64_t n, int group, int bits, const uint16_t* bias, int epilogue,
                const uint16_t* gate, const uint16_t* resid, const uint32_t* rowmap,
                uint16_t* y, uint16_t* y_raw);

/* h3_fused_rmsnorm_rope (网络算子-融合-RMSNormRoPE-通用.swift:41-94).
 * Row (s, h) of hd values at x[s*x_stride + h*hd]; cos/sin [S, rot/2]. */
int wxo_qk_norm_rope(const uint16_t* x, int64_t x_stride, int64_t S, int H, int hd,
                     const uint16_t* w, const uint16_t* cos_t, const uint16_t* sin_t,
                     int rot, float eps, uint16_t* out, int64_t out_stride);

/* h3_fused_norm_modscale (fused:133-168); rowmap NULL = every row uses mod row 0
 * (fusedNormModscaleRow, fused:295-315). */
int wxo_norm_modscale(const uint16_t* x, int64_t S, int64_t hidden, const uint16_t* w,
                      const uint16_t* shift, const uint16_t* scale, const uint32_t* rowmap,
                      float eps, uint16_t* out);

/* h3_fused_mod_gate (fused:179-196): out = bf16(x + other * gate[map[r]]) */
int wxo_mod_gate(const uint16_t* x, const uint16_t* other, const uint16_t* gate,
                 const uint32_t* rowmap, int64_t S, int64_t hidden, uint16_t* out);

/* SOL tau router (网络算子-稀疏注意力-SOL通用.swift:455-497), fixed fp32 order:
 *   qc/kc  = (sequential sum over the block's real rows) / len
 *   vsum   = sequential sum over rows (stored bf16)
 *   kMean  = (sequential sum over blocks) / nV; kcc = kc - kMean
 *   kcVar  = (sequential sum over blocks of kcc*kcc) / nV
 *   cm     = bf16( fma-chain_d(qc[d], kcc[d]) * scale )
 *   var    = sequential sum_d ((qc*qc)*kcVar); thr = tau * sqrt(var*(scale*scale) + 1e-6)
 *   sel    = (float(cm) > thr) || |qb-j| <= 1 || sink_start <= j < sink_end
 * q/k/v rows: x[s*row_stride + h*hd]; video rows are [g, S). */
int wxo_sol_route(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                  int64_t S, int H, int hd, int64_t g, int block, float scale, float tau,
                  int sink_start, int sink_end,
                  uint8_t* sel, float* thr, uint16_t* cm, uint16_t* vsum, float* lens);

/* Block top-k router (benchmark mode): score = fma-chain_d(qc, kc) * scale with
 * qc/kc block means as above (no centring); keep the diagonal plus the
 * ceil(density*nb) highest-scoring other blocks, ties to the lower index.
 * cm/vsum/lens are filled as in the SOL router (cm = bf16(score)). */
int wxo_topk_route(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                   int64_t S, int H, int hd, int64_t g, int block, float scale, float density,
                   uint8_t* sel, float* scores, uint16_t* cm, uint16_t* vsum, float* lens);

/* SOL attention semantics of h3sol_flash_v6 (SOL:110-231) with strip rows dense
 * (SOL:428-437). sel == NULL: dense attention for every row. Online softmax
 * in fp32; strip keys first, then video blocks in ascending order; selected
 * blocks exact, unselected blocks add the tail pooled term when tail != 0. */
int wxo_sparse_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                         int64_t S, int H, int hd, int64_t g, int block, float scale,
                         const uint8_t* sel, const uint16_t* cm, const uint16_t* vsum,
                         const float* lens, int tail, uint16_t* out, int64_t out_stride);

/* the same for query rows [row0, row1) only (bounded CPU-baseline samples);
 * out rows outside the range are not written */
int wxo_sparse_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t row_stride,
                              int64_t S, int H, int hd, int64_t g, int block, float scale,
                              const uint8_t* sel, const uint16_t* cm, const uint16_t* vsum,
                              const float* lens, int tail, int64_t row0, int64_t row1,
                              uint16_t* out, int64_t out_stride);

/* fp32 dense linear y[m][n] = sum_k x[m][k]*w[k][n] + b[n] (H3TensorOps.denseLinear,
 * the fp32 patch-embed / final-head islands, H3Transformer.swift:1036-1039, 1192-1203) */
int wxo_dense_f32(const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                  const float* b, float* y);

int wxo_num_threads(void);
/* OpenMP threads of later calls (n <= 0: every processor); returns the count now in force */
int wxo_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
