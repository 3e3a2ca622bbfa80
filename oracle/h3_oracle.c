/*
 * h3_oracle.c -- CPU restatement of the H3 self-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under minimax-h3-swift_b200/csrc.  Only tests/, the smoke() check in
 * __graft_entry__.py and the cpu_baseline / --impl reference legs of bench.py
 * load it.  The product path never calls it and has no CPU fallback.
 *
 * Parity status: PARTIAL.  The reference (MiniMax-H3-Swift) runs its dense
 * attention through MLXFast.scaledDotProductAttention (mlx-swift 0.31.6,
 * rev 0bb916c67f4b9e5c682cbe02a42c701c93ab5021), whose source is not vendored
 * and which cannot run in this container (no Swift, no MLX).  The in-tree
 * Swift semantics that this file restates are pinned by the reference's own
 * known-answer tests (ported in tests/test_oracle_*.py); MLX's accumulation
 * order is unpinned, so attention parity is stated as a tolerance
 * (max-abs <= 2e-2, mean-abs <= 2e-3 on unit-variance bf16 inputs).
 *
 * What each function follows (paths inside the reference project):
 *   h3o_rmsnorm_rows      Sources/H3Modules/Modulation.swift:116-120 (H3RMSNorm)
 *   h3o_rope_rows         Sources/H3Modules/DiTBlock.swift:83-103 (SplitHalfRoPE)
 *                         with the per-op bf16 rounding of
 *                         Tests/H3ModulesTests/QKFusionMetalFixture.swift:50-73
 *   h3o_rope_table        Sources/H3Modules/H3Transformer.swift:62-78 (H3RoPE),
 *                         with the per-axis theta split fixed by the benchmark
 *                         configuration (t/h/w = 32/48/48, theta 1e4)
 *   h3o_attend_streaming  Sources/H3Attention/AxialReference.swift:129-171
 *                         (online softmax: m0 = -3e38, masked = -1e30,
 *                         out = acc / max(l, 1e-30))
 *   h3o_attend_masked     Sources/H3Attention/AxialReference.swift:89-114
 *                         (one masked softmax per query row over the union)
 *   h3o_blockmask_*       the block-mask generator; it has no counterpart in
 *                         the reference and is defined by the benchmark
 *                         configuration plus AxialTopology's prefix rule
 *                         (Sources/H3Attention/AxialTopology.swift:128-137)
 *
 * All tensors are bf16 stored as uint16_t.  A q/k/v/o view is (pointer,
 * token stride, head stride) in elements with head_dim contiguous, so both
 * the [S,H,D] layout of AttentionLayer and the [H,S,D] layout of the backend
 * seam are expressible.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* round-to-nearest-even, NaN kept quiet */
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float rbf(float f) { return bf2f(f2bf(f)); }

void h3o_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}

void h3o_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]);
}

/* --------------------------------------------------------------- PRNG */

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

/* Counter-based N(0,1): element i of (seed, stream) is a pure function of the
 * three, so the device generator and this one produce the same bits.  Pair
 * p = i/2 draws one 64-bit word; Box-Muller in double, cos for even i, sin for
 * odd i; mean + std*z is rounded double -> float -> bf16. */
static inline double normal_at(uint64_t seed, uint64_t stream, uint64_t i) {
  uint64_t h = splitmix64(splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) + (i >> 1));
  double u1 = ((double)(h >> 40) + 1.0) * (1.0 / 16777216.0); /* (0,1] */
  double u2 = (double)(h & 0xFFFFFFull) * (1.0 / 16777216.0); /* [0,1) */
  double r = sqrt(-2.0 * log(u1));
  double a = 6.283185307179586 * u2;
  return (i & 1) ? r * sin(a) : r * cos(a);
}

void h3o_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream,
                          double mean, double std) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    out[i] = f2bf((float)(mean + std * normal_at(seed, stream, (uint64_t)i)));
}

/* ------------------------------------------------------- prologue (A2, A3) */

/* H3RMSNorm over head_dim for rows (token, head):
 *   f = fp32(x); n = f * rsqrt(mean(f*f) + eps); y = bf16(n * fp32(w))
 * Sum of squares accumulated in fp32 in index order. */
void h3o_rmsnorm_rows(const uint16_t* x, int64_t x_tok, int64_t x_head,
                      uint16_t* y, int64_t y_tok, int64_t y_head,
                      const uint16_t* w, int32_t seq_len, int32_t heads,
                      int32_t head_dim, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)seq_len * heads; ++r) {
    int64_t s = r / heads, h = r % heads;
    const uint16_t* xr = x + s * x_tok + h * x_head;
    uint16_t* yr = y + s * y_tok + h * y_head;
    float ss = 0.f;
    for (int d = 0; d < head_dim; ++d) {
      float f = bf2f(xr[d]);
      ss += f * f;
    }
    float inv = 1.0f / sqrtf(ss / (float)head_dim + eps);
    for (int d = 0; d < head_dim; ++d) yr[d] = f2bf((bf2f(xr[d]) * inv) * bf2f(w[d]));
  }
}

/* SplitHalfRoPE on bf16 rows, in place.  table is [S, half, 4] holding
 * (c, -s, s, c) per pair (i, i+half); channels >= 2*half pass through.
 * Every product and every sum is rounded to bf16, as MLX's bf16 elementwise
 * ops do. */
void h3o_rope_rows(uint16_t* x, int64_t x_tok, int64_t x_head, const uint16_t* table,
                   int32_t half, int32_t seq_len, int32_t heads) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)seq_len * heads; ++r) {
    int64_t s = r / heads, h = r % heads;
    uint16_t* xr = x + s * x_tok + h * x_head;
    const uint16_t* t = table + s * (int64_t)half * 4;
    for (int i = 0; i < half; ++i) {
      float c = bf2f(t[4 * i]), ns = bf2f(t[4 * i + 1]), sn = bf2f(t[4 * i + 2]),
            c2 = bf2f(t[4 * i + 3]);
      float a = bf2f(xr[i]), b = bf2f(xr[i + half]);
      float ra = rbf(rbf(c * a) + rbf(ns * b));
      float rb = rbf(rbf(sn * a) + rbf(c2 * b));
      xr[i] = f2bf(ra);
      xr[i + half] = f2bf(rb);
    }
  }
}

/* H3RoPE table for integer positions pos[S,3] (t, h, w).  Axis a has dims[a]
 * rotary channels, i.e. dims[a]/2 frequencies inv_k = theta^(-2k/dims[a])
 * (computed in double, stored as fp32 like a checkpoint's inv_freq).  The
 * first-half angles are cat(t*inv_t, h*inv_h, w*inv_w) in fp32; the table holds
 * bf16(fp32(cos)), bf16(-fp32(sin)), bf16(fp32(sin)), bf16(fp32(cos)), with
 * cos/sin evaluated in double on the fp32 angle. */
void h3o_rope_table(const int32_t* pos, int32_t seq_len, const int32_t* dims, double theta,
                    uint16_t* table) {
  int32_t half = (dims[0] + dims[1] + dims[2]) / 2;
  float inv[256];
  int n = 0;
  for (int a = 0; a < 3; ++a)
    for (int k = 0; k < dims[a] / 2; ++k)
      inv[n++] = (float)pow(theta, -2.0 * (double)k / (double)dims[a]);
#pragma omp parallel for schedule(static)
  for (int64_t s = 0; s < seq_len; ++s) {
    int i = 0;
    for (int a = 0; a < 3; ++a) {
      float p = (float)pos[s * 3 + a];
      for (int k = 0; k < dims[a] / 2; ++k, ++i) {
        float ang = p * inv[i];
        float c = (float)cos((double)ang), sn = (float)sin((double)ang);
        uint16_t* t = table + (s * half + i) * 4;
        t[0] = f2bf(c);
        t[1] = f2bf(-sn);
        t[2] = f2bf(sn);
        t[3] = f2bf(c);
      }
    }
  }
}

/* ------------------------------------------------------ block mask (A10) */

typedef struct {
  int32_t seq_len, block, prefix_len;
  int32_t frames, height, width;
  int32_t cell_t, cell_h, cell_w;
  int32_t radius_t, radius_h, radius_w;
  int32_t n_random;
  uint64_t seed;
} h3o_mask_spec;

static int mask_nblocks(const h3o_mask_spec* m) { return (m->seq_len + m->block - 1) / m->block; }

/* Coarse cell of block b, from the lattice coordinates of its first token.
 * Only meaningful for video blocks (first token >= prefix_len). */
static void block_cell(const h3o_mask_spec* m, int b, int* ct, int* ch, int* cw) {
  int64_t v = (int64_t)b * m->block - m->prefix_len;
  int64_t per = (int64_t)m->height * m->width;
  int t = (int)(v / per), rem = (int)(v % per);
  *ct = t / m->cell_t;
  *ch = (rem / m->width) / m->cell_h;
  *cw = (rem % m->width) / m->cell_w;
}

/* Kept flags of query block i, written to row[0..nb).  Rule:
 *   prefix query block (contains any prefix token)  -> every key block
 *   otherwise: prefix key blocks, the 3D-local window |dct|<=Rt, |dch|<=Rh,
 *   |dcw|<=Rw over video key blocks, then n_random distinct extra key blocks
 *   drawn by splitmix64 from state seed ^ (i * golden), candidate
 *   j = (hi32(word) * nb) >> 32, at most 64 + 16*n_random draws. */
static void mask_row(const h3o_mask_spec* m, int i, uint8_t* row) {
  int nb = mask_nblocks(m);
  int npb = (m->prefix_len + m->block - 1) / m->block; /* blocks touching the prefix */
  if (i < npb) {
    memset(row, 1, (size_t)nb);
    return;
  }
  memset(row, 0, (size_t)nb);
  for (int j = 0; j < npb && j < nb; ++j) row[j] = 1;
  int qt, qh, qw;
  block_cell(m, i, &qt, &qh, &qw);
  for (int j = npb; j < nb; ++j) {
    int kt, kh, kw;
    block_cell(m, j, &kt, &kh, &kw);
    if (abs(kt - qt) <= m->radius_t && abs(kh - qh) <= m->radius_h && abs(kw - qw) <= m->radius_w)
      row[j] = 1;
  }
  uint64_t state = m->seed ^ ((uint64_t)i * 0x9E3779B97F4A7C15ull);
  int added = 0, draws = 64 + 16 * m->n_random;
  for (int a = 0; a < draws && added < m->n_random; ++a) {
    state = splitmix64(state);
    int j = (int)(((state >> 32) * (uint64_t)nb) >> 32);
    if (!row[j]) {
      row[j] = 1;
      ++added;
    }
  }
}

/* Validates the spec; returns 0 if usable. */
int h3o_blockmask_check(const h3o_mask_spec* m) {
  if (m->seq_len <= 0 || m->block <= 0 || m->prefix_len < 0 || m->prefix_len > m->seq_len) return 1;
  if ((int64_t)m->frames * m->height * m->width != (int64_t)m->seq_len - m->prefix_len) return 2;
  if (m->cell_t <= 0 || m->cell_h <= 0 || m->cell_w <= 0) return 3;
  if (m->radius_t < 0 || m->radius_h < 0 || m->radius_w < 0 || m->n_random < 0) return 4;
  return 0;
}

/* CSR build.  col_idx may be NULL to query nnz only.  Returns spec status. */
int h3o_blockmask_build(const h3o_mask_spec* m, int32_t* row_ptr, int32_t* col_idx,
                        int64_t* nnz) {
  int st = h3o_blockmask_check(m);
  if (st) return st;
  int nb = mask_nblocks(m);
  uint8_t* row = (uint8_t*)malloc((size_t)nb);
  int64_t off = 0;
  if (row_ptr) row_ptr[0] = 0;
  for (int i = 0; i < nb; ++i) {
    mask_row(m, i, row);
    for (int j = 0; j < nb; ++j)
      if (row[j]) {
        if (col_idx) col_idx[off] = j;
        ++off;
      }
    if (row_ptr) row_ptr[i + 1] = (int32_t)off;
  }
  free(row);
  if (nnz) *nnz = off;
  return 0;
}

/* ------------------------------------------------------ attention (A8, A9) */

typedef struct {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  int64_t q_tok, q_head, k_tok, k_head, v_tok, v_head;
  float* out; /* fp32, [H, S, D] when out_f32 is set */
  uint16_t* out_bf16;
  int64_t o_tok, o_head; /* strides of out_bf16 */
  int32_t seq_len, heads, head_dim, block;
  float scale;
  const int32_t* row_ptr;
  const int32_t* col_idx;
} h3o_attn_args;

/* Online-softmax attention over the kept key blocks of each query block, in
 * ascending block order, one key tile per kept block (key columns past
 * seq_len inside the last block take the -1e30 sentinel).  Rows of query
 * blocks listed in qblocks (or all blocks if qblocks == NULL) for heads
 * [h0, h0 + hn) are computed.  fp32 throughout. */
void h3o_attend_streaming(const h3o_attn_args* a, const int32_t* qblocks, int32_t nqb,
                          int32_t h0, int32_t hn) {
  int nb = (a->seq_len + a->block - 1) / a->block;
  int nq = qblocks ? nqb : nb;
  int D = a->head_dim, B = a->block;
#pragma omp parallel
  {
    float* qf = (float*)malloc(sizeof(float) * B * D);
    float* kf = (float*)malloc(sizeof(float) * B * D);
    float* vf = (float*)malloc(sizeof(float) * B * D);
    float* acc = (float*)malloc(sizeof(float) * B * D);
    float* sc = (float*)malloc(sizeof(float) * B * B);
    float* mrow = (float*)malloc(sizeof(float) * B);
    float* lrow = (float*)malloc(sizeof(float) * B);
#pragma omp for schedule(dynamic, 1) collapse(2)
    for (int hh = 0; hh < hn; ++hh)
      for (int qi = 0; qi < nq; ++qi) {
        int h = h0 + hh;
        int ib = qblocks ? qblocks[qi] : qi;
        int r0 = ib * B, rows = a->seq_len - r0 < B ? a->seq_len - r0 : B;
        for (int r = 0; r < rows; ++r)
          for (int d = 0; d < D; ++d)
            qf[r * D + d] = bf2f(a->q[(int64_t)(r0 + r) * a->q_tok + (int64_t)h * a->q_head + d]);
        for (int r = 0; r < rows; ++r) {
          mrow[r] = -3e38f;
          lrow[r] = 0.f;
        }
        memset(acc, 0, sizeof(float) * B * D);
        for (int p = a->row_ptr[ib]; p < a->row_ptr[ib + 1]; ++p) {
          int jb = a->col_idx[p];
          int c0 = jb * B, cols = a->seq_len - c0 < B ? a->seq_len - c0 : B;
          for (int c = 0; c < cols; ++c)
            for (int d = 0; d < D; ++d) {
              kf[c * D + d] = bf2f(a->k[(int64_t)(c0 + c) * a->k_tok + (int64_t)h * a->k_head + d]);
              vf[c * D + d] = bf2f(a->v[(int64_t)(c0 + c) * a->v_tok + (int64_t)h * a->v_head + d]);
            }
          for (int r = 0; r < rows; ++r) {
            float tmax = -3e38f;
            for (int c = 0; c < B; ++c) {
              float s;
              if (c < cols) {
                s = 0.f;
                for (int d = 0; d < D; ++d) s += qf[r * D + d] * kf[c * D + d];
                s *= a->scale;
              } else {
                s = -1e30f;
              }
              sc[r * B + c] = s;
              if (s > tmax) tmax = s;
            }
            float mnew = mrow[r] > tmax ? mrow[r] : tmax;
            float resc = expf(mrow[r] - mnew);
            float lsum = 0.f;
            float* ar = acc + r * D;
            for (int d = 0; d < D; ++d) ar[d] *= resc;
            for (int c = 0; c < cols; ++c) {
              float pv = expf(sc[r * B + c] - mnew);
              lsum += pv;
              const float* vr = vf + c * D;
              for (int d = 0; d < D; ++d) ar[d] += pv * vr[d];
            }
            for (int c = cols; c < B; ++c) lsum += expf(sc[r * B + c] - mnew);
            lrow[r] = lrow[r] * resc + lsum;
            mrow[r] = mnew;
          }
        }
        for (int r = 0; r < rows; ++r) {
          float l = lrow[r] > 1e-30f ? lrow[r] : 1e-30f;
          for (int d = 0; d < D; ++d) {
            float o = acc[r * D + d] / l;
            if (a->out) a->out[((int64_t)h * a->seq_len + r0 + r) * D + d] = o;
            if (a->out_bf16)
              a->out_bf16[(int64_t)(r0 + r) * a->o_tok + (int64_t)h * a->o_head + d] = f2bf(o);
          }
        }
      }
    free(qf); free(kf); free(vf); free(acc); free(sc); free(mrow); free(lrow);
  }
}

/* The definition: for each query row one softmax over all S keys with an
 * additive mask of 0 (kept block pair) or -1e30 (dropped), max-subtracted,
 * in fp32.  Writes fp32 out[H,S,D].  O(S^2) memory-free but O(S^2 D) time:
 * for small cases only. */
void h3o_attend_masked(const h3o_attn_args* a) {
  int S = a->seq_len, D = a->head_dim, B = a->block;
  int nb = (S + B - 1) / B;
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * S);
    uint8_t* keep = (uint8_t*)malloc((size_t)nb);
#pragma omp for schedule(dynamic, 4) collapse(2)
    for (int h = 0; h < a->heads; ++h)
      for (int r = 0; r < S; ++r) {
        int ib = r / B;
        memset(keep, 0, (size_t)nb);
        for (int p = a->row_ptr[ib]; p < a->row_ptr[ib + 1]; ++p) keep[a->col_idx[p]] = 1;
        float mx = -3e38f;
        const uint16_t* qr = a->q + (int64_t)r * a->q_tok + (int64_t)h * a->q_head;
        for (int c = 0; c < S; ++c) {
          const uint16_t* kr = a->k + (int64_t)c * a->k_tok + (int64_t)h * a->k_head;
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += bf2f(qr[d]) * bf2f(kr[d]);
          s = s * a->scale + (keep[c / B] ? 0.f : -1e30f);
          sc[c] = s;
          if (s > mx) mx = s;
        }
        float l = 0.f;
        for (int c = 0; c < S; ++c) {
          sc[c] = expf(sc[c] - mx);
          l += sc[c];
        }
        for (int d = 0; d < D; ++d) {
          float o = 0.f;
          for (int c = 0; c < S; ++c)
            o += sc[c] * bf2f(a->v[(int64_t)c * a->v_tok + (int64_t)h * a->v_head + d]);
          a->out[((int64_t)h * S + r) * D + d] = o / l;
        }
      }
    free(sc);
    free(keep);
  }
}

int h3o_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void h3o_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* H3RoPE exactly as the reference builds it for the production model
 * (Sources/H3Modules/H3Transformer.swift:62-78): float positions pos[S,3]
 * (PackedLayout.positionIds, f64 cast to fp32), ONE shared inv_freq[n]
 * (from the checkpoint) applied to each of t, h, w; angles =
 * cat(t*inv, h*inv, w*inv) in fp32 (half = 3n); table entry =
 * (c, -s, s, c) of fp32 cos/sin (evaluated in double here) rounded to bf16. */
void h3o_rope_table_shared(const float* pos, int32_t seq_len, const float* inv, int32_t n, uint16_t* table) {
  const int32_t half = 3 * n;
#pragma omp parallel for schedule(static)
  for (int64_t s = 0; s < seq_len; ++s) {
    for (int a = 0; a < 3; ++a) {
      for (int k = 0; k < n; ++k) {
        float ang = pos[s * 3 + a] * inv[k];
        float c = (float)cos((double)ang), sn = (float)sin((double)ang);
        uint16_t* t = table + (s * half + a * n + k) * 4;
        t[0] = f2bf(c);
        t[1] = f2bf(-sn);
        t[2] = f2bf(sn);
        t[3] = f2bf(c);
      }
    }
  }
}
