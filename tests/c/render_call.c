/*
 * One render's attention call through the C ABI from plain C -- what a
 * Swift (CH3Cuda) or cgo binder does, with no Python or PyTorch involved.
 *
 *   render_call host            packed layout + host block list; prints a
 *                               summary line the tests compare
 *   render_call device OUT.bin  the same on cuda:0: inputs from the library's
 *                               generator, the RoPE table from the layout,
 *                               the block list built on the device, one fused
 *                               call; writes the bf16 output [S, H, 128]
 *
 * The render: 480x864, 5 s (124 frames), 332 text tokens, one keyframe at
 * frame 0 (the shape of tests/test_layout.py's render); H = 4 heads; mask
 * radius (1, 2, 2), 4 random blocks, seed 11; eps 1e-5; a shared 16-entry
 * inv_freq theta^(-k/16).  Device memory comes from the CUDA runtime.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "h3cuda.h"

#define HEADS 4

static int fail(const char* what, h3c_status st, h3c_ctx* ctx) {
  fprintf(stderr, "%s: status %d %s\n", what, (int)st, ctx ? h3c_last_error(ctx) : "");
  return 1;
}

static void render(h3c_layout_spec* spec, int32_t* keyframe) {
  memset(spec, 0, sizeof(*spec));
  spec->text_tokens = 332;
  spec->frame_count = 124; /* LatentGeometry(width: 864, height: 480, length: 120) */
  spec->latent_t = 37;
  spec->audio_t = 207;
  spec->latent_h = 30;
  spec->latent_w = 54;
  spec->patch = 2;
  keyframe[0] = 0;
  spec->n_keyframes = 1;
  spec->keyframes = keyframe;
}

static int mask_for(const h3c_layout_spec* spec, h3c_mask_spec* m, int64_t* total) {
  h3c_segment seg[8];
  int32_t nseg = 0;
  char err[256];
  if (h3c_packed_layout(spec, seg, 8, &nseg, total, err, sizeof(err)) != H3C_OK) {
    fprintf(stderr, "%s\n", err);
    return 1;
  }
  const h3c_segment* video = &seg[nseg - 1];
  if (video->kind != H3C_SEG_VIDEO || video->stop != *total) return 1;
  memset(m, 0, sizeof(*m));
  m->seq_len = (int32_t)*total;
  m->block = 128;
  m->prefix_len = video->start;
  m->frames = spec->latent_t;
  m->height = spec->latent_h / spec->patch;
  m->width = spec->latent_w / spec->patch;
  m->cell_t = 1;
  m->cell_h = 16;
  m->cell_w = 32;
  m->radius_t = 1;
  m->radius_h = 2;
  m->radius_w = 2;
  m->n_random = 4;
  m->seed = 11;
  printf("segments %d:", nseg);
  for (int i = 0; i < nseg; ++i) printf(" (%d,%d,%d)", seg[i].start, seg[i].stop, seg[i].kind);
  printf("\n");
  return 0;
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  int32_t keyframe[1];
  h3c_layout_spec spec;
  render(&spec, keyframe);
  h3c_mask_spec m;
  int64_t total = 0;
  if (mask_for(&spec, &m, &total)) return fail("h3c_packed_layout", H3C_ERR_INVALID_ARGUMENT, NULL);
  const int nb = (m.seq_len + 127) / 128;
  int64_t nnz = 0;
  h3c_status st = h3c_blockmask_build(&m, NULL, NULL, 0, &nnz);
  if (st != H3C_OK) return fail("h3c_blockmask_build (count)", st, NULL);
  int32_t* row_ptr = malloc(sizeof(int32_t) * (nb + 1));
  int32_t* col_idx = malloc(sizeof(int32_t) * nnz);
  st = h3c_blockmask_build(&m, row_ptr, col_idx, nnz, &nnz);
  if (st != H3C_OK) return fail("h3c_blockmask_build", st, NULL);
  uint64_t check = 0;
  for (int64_t i = 0; i < nnz; ++i) check = check * 1000003u + (uint64_t)col_idx[i];
  printf("abi %d total %lld prefix %d blocks %d nnz %lld check %llu\n", h3c_abi_version(), (long long)total,
         m.prefix_len, nb, (long long)nnz, (unsigned long long)check);
  if (strcmp(argv[1], "host") == 0) return 0;
  if (strcmp(argv[1], "device") != 0 || argc < 3) return 2;

  /* ---------------------------------------------------------------- device */
  h3c_ctx* ctx = NULL;
  if ((st = h3c_init(0, &ctx)) != H3C_OK) return fail("h3c_init", st, ctx);
  const int64_t S = total, n = S * HEADS * 128;
  void *q, *k, *v, *o, *wq, *wk, *inv, *table;
  int32_t *d_rp, *d_ci;
  if (cudaMalloc(&q, n * 2) || cudaMalloc(&k, n * 2) || cudaMalloc(&v, n * 2) || cudaMalloc(&o, n * 2) ||
      cudaMalloc(&wq, 256) || cudaMalloc(&wk, 256) || cudaMalloc(&inv, 16 * 4) || cudaMalloc(&table, S * 48 * 8) ||
      cudaMalloc((void**)&d_rp, 4 * (nb + 1)) || cudaMalloc((void**)&d_ci, 4 * nnz))
    return fail("cudaMalloc", H3C_ERR_CUDA, NULL);
  /* the same generator streams as the Python tests: seed 41, streams 1..5 */
  if ((st = h3c_fill_normal_bf16(ctx, q, n, 41, 1, 0.0, 1.0, NULL)) != H3C_OK ||
      (st = h3c_fill_normal_bf16(ctx, k, n, 41, 2, 0.0, 1.0, NULL)) != H3C_OK ||
      (st = h3c_fill_normal_bf16(ctx, v, n, 41, 3, 0.0, 1.0, NULL)) != H3C_OK ||
      (st = h3c_fill_normal_bf16(ctx, wq, 128, 41, 4, 1.0, 0.02, NULL)) != H3C_OK ||
      (st = h3c_fill_normal_bf16(ctx, wk, 128, 41, 5, 1.0, 0.02, NULL)) != H3C_OK)
    return fail("h3c_fill_normal_bf16", st, ctx);
  float inv_h[16];
  for (int i = 0; i < 16; ++i) inv_h[i] = (float)pow(1e4, -(double)i / 16.0);
  if (cudaMemcpy(inv, inv_h, sizeof(inv_h), cudaMemcpyHostToDevice)) return fail("cudaMemcpy", H3C_ERR_CUDA, NULL);
  if ((st = h3c_rope_table_layout(ctx, &spec, (const float*)inv, 16, table, S, NULL)) != H3C_OK)
    return fail("h3c_rope_table_layout", st, ctx);
  int64_t nnz_d = 0;
  if ((st = h3c_blockmask_build_device(ctx, &m, d_rp, d_ci, nnz, &nnz_d, NULL)) != H3C_OK)
    return fail("h3c_blockmask_build_device", st, ctx);
  if (nnz_d != nnz) return fail("device block list size", H3C_ERR_INVALID_ARGUMENT, ctx);

  h3c_attn_args a;
  memset(&a, 0, sizeof(a));
  const h3c_view vq = {q, HEADS * 128, 128}, vk = {k, HEADS * 128, 128}, vv = {v, HEADS * 128, 128},
                 vo = {o, HEADS * 128, 128};
  a.q = vq;
  a.k = vk;
  a.v = vv;
  a.out = vo;
  a.seq_len = (int32_t)S;
  a.heads = HEADS;
  a.head_dim = 128;
  a.head_offset = 0;
  a.head_count = HEADS;
  a.scale = 1.0f / sqrtf(128.0f);
  a.row_ptr = d_rp;
  a.col_idx = d_ci;
  a.block = 128;
  a.flags = H3C_FUSE_PROLOGUE;
  a.q_norm_weight = wq;
  a.k_norm_weight = wk;
  a.eps = 1e-5f;
  a.rope_table = table;
  a.rope_half = 48;
  if ((st = h3c_attn_fwd_sync(ctx, &a, NULL)) != H3C_OK) return fail("h3c_attn_fwd_sync", st, ctx);
  uint16_t* out = malloc(n * 2);
  if (cudaMemcpy(out, o, n * 2, cudaMemcpyDeviceToHost)) return fail("cudaMemcpy", H3C_ERR_CUDA, NULL);
  FILE* f = fopen(argv[2], "wb");
  if (!f || fwrite(out, 2, n, f) != (size_t)n) return fail("write", H3C_ERR_INVALID_ARGUMENT, NULL);
  fclose(f);
  printf("device ok\n");
  h3c_destroy(ctx);
  return 0;
}
