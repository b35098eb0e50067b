// wx_graph.cu — one DiT block forward captured as a CUDA graph and replayed.
//
// A block issues ~12-20 kernels (norm, projections with their weight expansion, routing,
// the attention kernels on the context stream and a side stream, the MLP); at small
// sizes (benchmark config 1: S = 4096) the gaps between dependent launches are a visible
// part of the block's time. The graph is captured once from wx_dit_block_forward on a
// private stream (relaxed capture mode: the kernel-attribute and occupancy queries the
// launch path makes on first use are host calls) and replayed on the context stream;
// every pointer is baked in, so the caller refreshes the buffers' contents between
// replays. Profiling and tracing are off while capturing (their events would be baked in).
#include <cuda_runtime.h>

#include "wx_internal.h"

struct wx_graph {
  cudaGraphExec_t exec = nullptr;
  int64_t kernels = 0;  // libwx kernels per replay
  int device = 0;
};

using namespace wx;

extern "C" {

int wx_dit_block_graph_create(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                              const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S,
                              const void* cos_t, const void* sin_t, const wx_sparse_spec* spec, void* pab_slot,
                              int refresh, void* scratch, wx_graph** out) {
  WX_CHECK_ARG(ctx, ctx && out);
  *out = nullptr;
  if (ctx->sp_size != 1)  // the sequence-parallel block waits on other ranks: not a replayable graph
    return set_error(ctx, WX_ERR_UNSUPPORTED, "block graphs are single-GPU (this context has %d ranks)",
                     ctx->sp_size);
  WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));  // nothing of the caller's is in flight
  cudaStream_t cap = nullptr;
  WX_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
  cudaStream_t saved = ctx->stream;
  const bool saved_prof = ctx->prof, saved_trace = ctx->trace;
  const int64_t l0 = ctx->launches;
  ctx->stream = cap;
  ctx->prof = false;
  ctx->trace = false;
  cudaGraph_t g = nullptr;
  int st = WX_OK;
  cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed);
  if (e == cudaSuccess) {
    st = wx_dit_block_forward(ctx, cfg, w, mods, rowmap, h, S, cos_t, sin_t, spec, pab_slot, refresh, scratch);
    e = cudaStreamEndCapture(cap, &g);  // ends the capture on every path
  }
  const int64_t captured = ctx->launches - l0;
  ctx->launches = l0;  // captured, not run
  ctx->stream = saved;
  ctx->prof = saved_prof;
  ctx->trace = saved_trace;
  cudaGraphExec_t ex = nullptr;
  if (st == WX_OK && e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(cap);
  if (st != WX_OK) {
    if (ex) cudaGraphExecDestroy(ex);
    return st;
  }
  if (e != cudaSuccess)
    return set_error(ctx, WX_ERR_CUDA, "block graph capture: %s", cudaGetErrorString(e));
  wx_graph* gr = new wx_graph();
  gr->exec = ex;
  gr->kernels = captured;
  gr->device = ctx->device;
  *out = gr;
  return WX_OK;
}

int wx_graph_launch(wx_ctx* ctx, wx_graph* g) {
  WX_CHECK_ARG(ctx, ctx && g && g->exec && g->device == ctx->device);
  WX_CUDA_TRY(ctx, cudaGraphLaunch(g->exec, ctx->stream));
  ctx->launches += g->kernels;
  return WX_OK;
}

int64_t wx_graph_kernels(const wx_graph* g) { return g ? g->kernels : -1; }

int wx_graph_destroy(wx_graph* g) {
  if (!g) return WX_OK;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  delete g;
  return WX_OK;
}

}  // extern "C"
