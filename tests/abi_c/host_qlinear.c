/* A host program that drives libwx through its C ABI alone (no Python, no CUDA runtime
 * calls of its own), as the reference's Swift host would through the module map:
 * wx_ctx_create -> wx_alloc / wx_upload -> wx_qlinear -> wx_download -> wx_ctx_check_device
 * -> wx_free -> wx_ctx_destroy.
 *
 *   host_qlinear M K N in.bin out.bin
 *
 * in.bin: x [M,K] bf16 | wq [N, K*6/32] u32 | scales [N, K/64] bf16 | biases [N, K/64] bf16 |
 *         bias [N] bf16 (raw little-endian); out.bin: y [M,N] bf16. Exit status 0 on success;
 * on failure the status and wx_last_error go to stderr. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "wx_api.h"

static int fail(wx_ctx* ctx, const char* what, int st) {
  fprintf(stderr, "%s: status %d: %s\n", what, st, ctx ? wx_last_error(ctx) : "");
  return 1;
}

int main(int argc, char** argv) {
  if (argc != 6) {
    fprintf(stderr, "usage: %s M K N in.bin out.bin\n", argv[0]);
    return 2;
  }
  const int64_t m = atoll(argv[1]), k = atoll(argv[2]), n = atoll(argv[3]);
  const size_t bx = (size_t)(m * k * 2), bw = (size_t)(n * k * 6 / 32 * 4), bs = (size_t)(n * (k / 64) * 2),
               bb = (size_t)(n * 2), by = (size_t)(m * n * 2);
  const size_t total = bx + bw + 2 * bs + bb;
  unsigned char* in = (unsigned char*)malloc(total);
  unsigned char* out = (unsigned char*)malloc(by);
  FILE* f = fopen(argv[4], "rb");
  if (!in || !out || !f || fread(in, 1, total, f) != total) {
    fprintf(stderr, "cannot read %zu bytes from %s\n", total, argv[4]);
    return 2;
  }
  fclose(f);
  wx_ctx* ctx = NULL;
  int st = wx_ctx_create(0, &ctx);
  if (st != WX_OK) return fail(NULL, "wx_ctx_create", st);
  void *dx = NULL, *dw = NULL, *ds = NULL, *dbi = NULL, *db = NULL, *dy = NULL;
  if ((st = wx_alloc(ctx, bx, &dx)) || (st = wx_alloc(ctx, bw, &dw)) || (st = wx_alloc(ctx, bs, &ds)) ||
      (st = wx_alloc(ctx, bs, &dbi)) || (st = wx_alloc(ctx, bb, &db)) || (st = wx_alloc(ctx, by, &dy)))
    return fail(ctx, "wx_alloc", st);
  size_t off = 0;
  if ((st = wx_upload(ctx, dx, in + off, bx))) return fail(ctx, "wx_upload x", st);
  off += bx;
  if ((st = wx_upload(ctx, dw, in + off, bw))) return fail(ctx, "wx_upload wq", st);
  off += bw;
  if ((st = wx_upload(ctx, ds, in + off, bs))) return fail(ctx, "wx_upload scales", st);
  off += bs;
  if ((st = wx_upload(ctx, dbi, in + off, bs))) return fail(ctx, "wx_upload biases", st);
  off += bs;
  if ((st = wx_upload(ctx, db, in + off, bb))) return fail(ctx, "wx_upload bias", st);
  wx_qweight w = {(const uint32_t*)dw, ds, dbi, db, n, k, 64, 6};
  if ((st = wx_qlinear(ctx, dx, m, k, &w, WX_EPI_NONE, NULL, NULL, NULL, dy, n, NULL)))
    return fail(ctx, "wx_qlinear", st);
  if ((st = wx_download(ctx, out, dy, by))) return fail(ctx, "wx_download", st);
  if ((st = wx_ctx_check_device(ctx))) return fail(ctx, "wx_ctx_check_device", st);
  void* bufs[6] = {dx, dw, ds, dbi, db, dy};
  for (int i = 0; i < 6; ++i)
    if ((st = wx_free(ctx, bufs[i]))) return fail(ctx, "wx_free", st);
  wx_ctx_destroy(ctx);
  f = fopen(argv[5], "wb");
  if (!f || fwrite(out, 1, by, f) != by) {
    fprintf(stderr, "cannot write %s\n", argv[5]);
    return 2;
  }
  fclose(f);
  free(in);
  free(out);
  return 0;
}
