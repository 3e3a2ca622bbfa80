// Small kernels around the attention: the Q/K prologue (RMSNorm + split-half
// RoPE), the RoPE table, the block-mask builder and the synthetic-input
// generator.  All are HBM- or latency-bound; the attention kernels are where
// the time goes.
#include "common.cuh"

namespace h3 {
namespace {

// ---------------------------------------------------------------- prologue
// 16 threads per (token, head) row of 128 channels, 8 contiguous channels
// (one 16-byte load) per thread, 16 rows per 256-thread CTA.  RMSNorm follows
// Sources/H3Modules/Modulation.swift:116-120 (fp32 sum of squares, fp32
// products, bf16 result); the rotation follows
// Sources/H3Modules/DiTBlock.swift:83-103 with each product and sum rounded
// to bf16 as in Tests/H3ModulesTests/QKFusionMetalFixture.swift:57-69.  The
// normalised row is staged in shared memory because the rotation pairs
// channel i with i + half for any half <= 64.
__global__ void __launch_bounds__(256) prologue_kernel(const uint16_t* __restrict__ x, int64_t x_tok,
                                                       int64_t x_head, uint16_t* __restrict__ y, int64_t y_tok,
                                                       int64_t y_head, int32_t seq_len, int32_t head_count,
                                                       const uint16_t* __restrict__ w, float eps,
                                                       const uint16_t* __restrict__ table, int32_t half) {
  __shared__ float rowbuf[16][129];
  const int sub = threadIdx.x >> 4, t = threadIdx.x & 15;
  const int64_t row = (int64_t)blockIdx.x * 16 + sub;
  const bool live = row < (int64_t)seq_len * head_count;
  const int64_t s = live ? row / head_count : 0, h = live ? row % head_count : 0;
  float v[8];
  float ss = 0.f;
  if (live) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + s * x_tok + h * x_head + 8 * t);
    const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(wv[i] << 16);
      v[2 * i + 1] = __uint_as_float(wv[i] & 0xffff0000u);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float inv = 1.0f / sqrtf(ss / 128.f + eps);
  const uint4 wraw = *reinterpret_cast<const uint4*>(w + 8 * t);
  const uint32_t ww[4] = {wraw.x, wraw.y, wraw.z, wraw.w};
  float* rb = rowbuf[sub];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float wi = __uint_as_float(i & 1 ? (ww[i >> 1] & 0xffff0000u) : (ww[i >> 1] << 16));
    rb[8 * t + i] = rbf((v[i] * inv) * wi);
  }
  __syncwarp();
  if (!live) return;
  const uint16_t* tr = table ? table + s * (int64_t)half * 4 : nullptr;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float r2[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int d = 8 * t + i + k;
      float out = rb[d];
      if (tr && d < 2 * half) {
        const int p = d < half ? d : d - half;
        const uint2 e = *reinterpret_cast<const uint2*>(tr + 4 * p);  // (c, -s, s, c)
        if (d < half) {
          const float c = __uint_as_float(e.x << 16), ns = __uint_as_float(e.x & 0xffff0000u);
          out = rbf(rbf(c * rb[d]) + rbf(ns * rb[d + half]));
        } else {
          const float sn = __uint_as_float(e.y << 16), c2 = __uint_as_float(e.y & 0xffff0000u);
          out = rbf(rbf(sn * rb[p]) + rbf(c2 * rb[d]));
        }
      }
      r2[k] = out;
    }
    o[i >> 1] = (uint32_t)f2bf(r2[0]) | ((uint32_t)f2bf(r2[1]) << 16);
  }
  *reinterpret_cast<uint4*>(y + s * y_tok + h * y_head + 8 * t) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Specialisation for any half that is a multiple of 4 (the benchmark's
// half 64, the production model's half 48) and for RMSNorm alone.  Every
// thread of the 16 on a row holds 8 channels: thread t < half/4 owns the
// rotation pairs 4t..4t+3 (channels 4t..4t+3 and half+4t..half+4t+3), the
// other threads own 8 contiguous pass-through channels from 2*half up, so
// each pair and its table entries stay in registers.  Same arithmetic as
// prologue_kernel, with the rotation on packed bf16x2 operations.

__device__ __forceinline__ void unpack4(uint2 u, float* f) {
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xffff0000u);
}


__global__ void __launch_bounds__(256) prologue_pairs_kernel(const uint16_t* __restrict__ x, int64_t x_tok,
                                                             int64_t x_head, uint16_t* __restrict__ y, int64_t y_tok,
                                                             int64_t y_head, int32_t seq_len, int32_t head_count,
                                                             const uint16_t* __restrict__ w, float eps,
                                                             const uint16_t* __restrict__ table, int32_t half) {
  const int sub = threadIdx.x >> 4, t = threadIdx.x & 15;
  const int64_t row = (int64_t)blockIdx.x * 16 + sub;
  const bool live = row < (int64_t)seq_len * head_count;
  const int64_t s = live ? row / head_count : 0, h = live ? row % head_count : 0;
  const bool pair = 4 * t < half;
  // channel offsets of this thread's two groups of 4
  const int ca = pair ? 4 * t : 2 * half + 8 * (t - half / 4);
  const int cb = pair ? half + 4 * t : ca + 4;
  float a[4], b[4], wa[4], wb[4];
  float ss = 0.f;
  const uint16_t* xr = x + s * x_tok + h * x_head;
  if (live) {
    unpack4(*reinterpret_cast<const uint2*>(xr + ca), a);
    unpack4(*reinterpret_cast<const uint2*>(xr + cb), b);
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += a[i] * a[i] + b[i] * b[i];
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  if (!live) return;
  const float inv = 1.0f / sqrtf(ss / 128.f + eps);
  unpack4(*reinterpret_cast<const uint2*>(w + ca), wa);
  unpack4(*reinterpret_cast<const uint2*>(w + cb), wb);
  // normalised values as bf16x2 words: A[k] = channels ca+2k, ca+2k+1;
  // B[k] = channels cb+2k, cb+2k+1 (the rotation partners of A[k] on a pair thread)
  __nv_bfloat162 A[2], B[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    A[k] = __floats2bfloat162_rn((a[2 * k] * inv) * wa[2 * k], (a[2 * k + 1] * inv) * wa[2 * k + 1]);
    B[k] = __floats2bfloat162_rn((b[2 * k] * inv) * wb[2 * k], (b[2 * k + 1] * inv) * wb[2 * k + 1]);
  }
  if (table && pair) {
    // Each product and each sum rounded to bf16 once: bf16 x bf16 is exact
    // in fp32, and where fp32 would round a sum of two bf16 values the bf16
    // result is the larger operand either way, so the packed bf16 ops (no
    // contraction) equal the fp32-then-round steps of the reference.
    const uint4* tp = reinterpret_cast<const uint4*>(table + (s * half + 4 * t) * 4);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint4 e = tp[k];  // entries 4t+2k and 4t+2k+1: (c, -s, s, c) each
      const uint32_t cw = __byte_perm(e.x, e.z, 0x5410), nsw = __byte_perm(e.x, e.z, 0x7632);
      const uint32_t sw = __byte_perm(e.y, e.w, 0x5410), c2w = __byte_perm(e.y, e.w, 0x7632);
      const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&cw);
      const __nv_bfloat162 ns = *reinterpret_cast<const __nv_bfloat162*>(&nsw);
      const __nv_bfloat162 sn = *reinterpret_cast<const __nv_bfloat162*>(&sw);
      const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162*>(&c2w);
      const __nv_bfloat162 ra = __hadd2_rn(__hmul2_rn(c, A[k]), __hmul2_rn(ns, B[k]));
      const __nv_bfloat162 rbv = __hadd2_rn(__hmul2_rn(sn, A[k]), __hmul2_rn(c2, B[k]));
      A[k] = ra;
      B[k] = rbv;
    }
  }
  uint16_t* yr = y + s * y_tok + h * y_head;
  *reinterpret_cast<uint2*>(yr + ca) =
      make_uint2(*reinterpret_cast<uint32_t*>(&A[0]), *reinterpret_cast<uint32_t*>(&A[1]));
  *reinterpret_cast<uint2*>(yr + cb) =
      make_uint2(*reinterpret_cast<uint32_t*>(&B[0]), *reinterpret_cast<uint32_t*>(&B[1]));
}

// Both operands of the fused call in one launch.  A warp owns one operand
// (its norm weights stay in registers) and walks tokens; for each token it
// loads the token's RoPE table entries once into registers and then
// normalises and rotates every head of that token, four rows at a time
// (8 threads per 128-channel row, two 16-byte loads and stores per thread,
// two heads in flight per thread).  Thread t of a row owns the rotation
// pairs 8t..8t+7 (channels 8t.. and half+8t..) when 8t < half, else 16
// contiguous pass-through channels from 2*half up; half must be a multiple
// of 8 (64 for the benchmark, 48 for the production model) and the table
// 16-byte aligned.  Arithmetic as prologue_pairs_kernel.
struct ProOperand {
  const uint16_t* x;
  int64_t x_tok, x_head;
  uint16_t* y;
  int64_t y_tok, y_head;
  const uint16_t* w;
};

__device__ __forceinline__ void unpack8(uint4 u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int U>
__global__ void __launch_bounds__(256, 3) prologue_qk_kernel(ProOperand op0, ProOperand op1, int32_t seq_len,
                                                             int32_t head_count, float eps,
                                                             const uint16_t* __restrict__ table, int32_t half) {
  // PDL: the dependent attention kernel may be scheduled as SMs free up; it
  // waits for this grid's completion before it reads the normalised rows
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, grp = lane >> 3, t = lane & 7;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;  // even: 8 warps per CTA
  // field by field: a reference to either parameter would put both in local memory
  const bool second = gw & 1;
  const uint16_t* __restrict__ px = second ? op1.x : op0.x;
  uint16_t* __restrict__ py = second ? op1.y : op0.y;
  const int64_t x_tok = second ? op1.x_tok : op0.x_tok, x_head = second ? op1.x_head : op0.x_head;
  const int64_t y_tok = second ? op1.y_tok : op0.y_tok, y_head = second ? op1.y_head : op0.y_head;
  const uint16_t* pw = second ? op1.w : op0.w;
  const bool rot = table != nullptr && 8 * t < half;
  const int hh = table ? half : 0;
  const int ca = rot ? 8 * t : 2 * hh + 16 * (t - hh / 8);
  const int cb = rot ? half + 8 * t : ca + 8;
  const uint4 wpa = *reinterpret_cast<const uint4*>(pw + ca), wpb = *reinterpret_cast<const uint4*>(pw + cb);

  for (int64_t s = gw >> 1; s < seq_len; s += nw >> 1) {
    // the token's rotation entries (c, -s, s, c) for pairs 8t..8t+7; read
    // per row (L1 hits after the token's first head)
    const uint4* tp = rot ? reinterpret_cast<const uint4*>(table + (s * half + 8 * t) * 4) : nullptr;
    const uint16_t* xs = px + s * x_tok;
    uint16_t* ys = py + s * y_tok;
    for (int h0 = grp; h0 < head_count; h0 += 4 * U) {
      // U heads per thread in flight: h0, h0 + 4, ...
      uint4 ra[U], rb[U];
      bool live[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int h = h0 + 4 * u;
        live[u] = h < head_count;
        if (live[u]) {
          const uint16_t* xr = xs + h * x_head;
          ra[u] = __ldcs(reinterpret_cast<const uint4*>(xr + ca));
          rb[u] = __ldcs(reinterpret_cast<const uint4*>(xr + cb));
        } else {
          ra[u] = rb[u] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float a[8], b[8];
        unpack8(ra[u], a);
        unpack8(rb[u], b);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += a[i] * a[i] + b[i] * b[i];
        ss += __shfl_xor_sync(0xffffffff, ss, 4);
        ss += __shfl_xor_sync(0xffffffff, ss, 2);
        ss += __shfl_xor_sync(0xffffffff, ss, 1);
        if (!live[u]) continue;
        const float inv = 1.0f / sqrtf(ss / 128.f + eps);
        float wa[8], wb[8];
        unpack8(wpa, wa);
        unpack8(wpb, wb);
        uint32_t A[4], B[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          A[k] = pack2((a[2 * k] * inv) * wa[2 * k], (a[2 * k + 1] * inv) * wa[2 * k + 1]);
          B[k] = pack2((b[2 * k] * inv) * wb[2 * k], (b[2 * k + 1] * inv) * wb[2 * k + 1]);
        }
        if (rot) {
          // each product and each sum rounded to bf16 once (see
          // prologue_pairs_kernel for why the packed bf16 ops are exact);
          // tp[k] holds the entries of pairs 8t+2k and 8t+2k+1
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 ek = tp[k];
            const uint32_t cw = __byte_perm(ek.x, ek.z, 0x5410), nsw = __byte_perm(ek.x, ek.z, 0x7632);
            const uint32_t sw = __byte_perm(ek.y, ek.w, 0x5410), c2w = __byte_perm(ek.y, ek.w, 0x7632);
            const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&cw);
            const __nv_bfloat162 ns = *reinterpret_cast<const __nv_bfloat162*>(&nsw);
            const __nv_bfloat162 sn = *reinterpret_cast<const __nv_bfloat162*>(&sw);
            const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162*>(&c2w);
            const __nv_bfloat162 av = *reinterpret_cast<const __nv_bfloat162*>(&A[k]);
            const __nv_bfloat162 bv = *reinterpret_cast<const __nv_bfloat162*>(&B[k]);
            const __nv_bfloat162 r0 = __hadd2_rn(__hmul2_rn(c, av), __hmul2_rn(ns, bv));
            const __nv_bfloat162 r1 = __hadd2_rn(__hmul2_rn(sn, av), __hmul2_rn(c2, bv));
            A[k] = *reinterpret_cast<const uint32_t*>(&r0);
            B[k] = *reinterpret_cast<const uint32_t*>(&r1);
          }
        }
        uint16_t* yr = ys + (h0 + 4 * u) * y_head;
        *reinterpret_cast<uint4*>(yr + ca) = make_uint4(A[0], A[1], A[2], A[3]);
        *reinterpret_cast<uint4*>(yr + cb) = make_uint4(B[0], B[1], B[2], B[3]);
      }
    }
  }
}

// -------------------------------------------------------------- rope table
// Follows H3RoPE.angles / rotationTable (Sources/H3Modules/H3Transformer.swift:62-78):
// fp32 inv_freq, fp32 angle = pos * inv, cos/sin evaluated in double on the
// fp32 angle and rounded to fp32 then bf16; entry = (c, -s, s, c).
__global__ void rope_table_kernel(const int32_t* __restrict__ pos, int32_t seq_len, int3 dims,
                                  const float* __restrict__ inv, int32_t half, uint16_t* __restrict__ table) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)seq_len * half) return;
  int64_t s = idx / half;
  int i = (int)(idx % half);
  int axis = i < dims.x / 2 ? 0 : (i < (dims.x + dims.y) / 2 ? 1 : 2);
  float p = (float)pos[s * 3 + axis];
  float ang = __fmul_rn(p, inv[i]);
  float c = (float)cos((double)ang), sn = (float)sin((double)ang);
  uint16_t* t = table + idx * 4;
  t[0] = f2bf(c);
  t[1] = f2bf(-sn);
  t[2] = f2bf(sn);
  t[3] = f2bf(c);
}

// Production table: float positions, one inv_freq vector shared by the
// three axes (H3RoPE.angles, Sources/H3Modules/H3Transformer.swift:62-68).
__global__ void rope_table_shared_kernel(const float* __restrict__ pos, int32_t seq_len,
                                         const float* __restrict__ inv, int32_t n, uint16_t* __restrict__ table) {
  const int32_t half = 3 * n;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)seq_len * half) return;
  int64_t s = idx / half;
  int i = (int)(idx % half);
  int axis = i / n;
  float ang = __fmul_rn(pos[s * 3 + axis], inv[i - axis * n]);
  float c = (float)cos((double)ang), sn = (float)sin((double)ang);
  uint16_t* t = table + idx * 4;
  t[0] = f2bf(c);
  t[1] = f2bf(-sn);
  t[2] = f2bf(sn);
  t[3] = f2bf(c);
}

// ------------------------------------------------------------- block mask
// One CTA per query block: a shared bitmap of kept key blocks, then the
// ascending column list.  Pass 0 writes row counts; pass 1 (after a
// single-CTA exclusive scan) writes col_idx.  Rule identical to the host
// builder in api.cu.
struct MaskDev {
  int32_t seq_len, block, prefix_len, frames, height, width, cell_t, cell_h, cell_w, radius_t, radius_h,
      radius_w, n_random;
  uint64_t seed;
  int32_t nb, npb;
};

__device__ __forceinline__ void cell_of(const MaskDev& m, int b, int& ct, int& ch, int& cw) {
  int64_t v = (int64_t)b * m.block - m.prefix_len;
  int64_t per = (int64_t)m.height * m.width;
  int t = (int)(v / per), rem = (int)(v % per);
  ct = t / m.cell_t;
  ch = (rem / m.width) / m.cell_h;
  cw = (rem % m.width) / m.cell_w;
}

__global__ void mask_rows_kernel(MaskDev m, int32_t* __restrict__ counts, const int32_t* __restrict__ row_ptr,
                                 int32_t* __restrict__ col_idx, int64_t capacity, int pass) {
  extern __shared__ uint32_t bits[];
  const int i = blockIdx.x;
  const int words = (m.nb + 31) / 32;
  const bool dense = i < m.npb;
  for (int wd = threadIdx.x; wd < words; wd += blockDim.x) bits[wd] = 0;
  __syncthreads();
  if (dense) {
    for (int j = threadIdx.x; j < m.nb; j += blockDim.x) atomicOr(&bits[j >> 5], 1u << (j & 31));
  } else {
    int qt, qh, qw;
    cell_of(m, i, qt, qh, qw);
    for (int j = threadIdx.x; j < m.nb; j += blockDim.x) {
      bool keep = j < m.npb;
      if (!keep) {
        int kt, kh, kw;
        cell_of(m, j, kt, kh, kw);
        keep = abs(kt - qt) <= m.radius_t && abs(kh - qh) <= m.radius_h && abs(kw - qw) <= m.radius_w;
      }
      if (keep) atomicOr(&bits[j >> 5], 1u << (j & 31));
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // the draws are sequential by definition
      uint64_t state = m.seed ^ ((uint64_t)i * 0x9E3779B97F4A7C15ull);
      int added = 0, draws = 64 + 16 * m.n_random;
      for (int a = 0; a < draws && added < m.n_random; ++a) {
        state = splitmix64(state);
        int j = (int)(((state >> 32) * (uint64_t)m.nb) >> 32);
        if (!(bits[j >> 5] & (1u << (j & 31)))) {
          bits[j >> 5] |= 1u << (j & 31);
          ++added;
        }
      }
    }
  }
  __syncthreads();
  if (pass == 0) {
    __shared__ int total;
    if (threadIdx.x == 0) total = 0;
    __syncthreads();
    int c = 0;
    for (int wd = threadIdx.x; wd < words; wd += blockDim.x) c += __popc(bits[wd]);
    atomicAdd(&total, c);
    __syncthreads();
    if (threadIdx.x == 0) counts[i] = total;
    return;
  }
  // pass 1: thread 0 walks the bitmap in order (nb <= a few thousand)
  if (threadIdx.x == 0) {
    int64_t off = row_ptr[i];
    for (int wd = 0; wd < words; ++wd) {
      uint32_t b = bits[wd];
      while (b) {
        int j = wd * 32 + __ffs(b) - 1;
        b &= b - 1;
        if (off < capacity) col_idx[off] = j;
        ++off;
      }
    }
  }
}

__global__ void scan_kernel(const int32_t* __restrict__ counts, int32_t nb, int32_t* __restrict__ row_ptr,
                            int64_t* __restrict__ nnz) {
  // single CTA, sequential chunks: nb is at most tens of thousands
  __shared__ int64_t part[1024];
  const int t = threadIdx.x, n = blockDim.x;
  const int chunk = (nb + n - 1) / n;
  int64_t sum = 0;
  for (int i = t * chunk; i < min(nb, (t + 1) * chunk); ++i) sum += counts[i];
  part[t] = sum;
  __syncthreads();
  if (t == 0) {
    int64_t run = 0;
    for (int i = 0; i < n; ++i) {
      int64_t v = part[i];
      part[i] = run;
      run += v;
    }
    *nnz = run;
  }
  __syncthreads();
  int64_t run = part[t];
  for (int i = t * chunk; i < min(nb, (t + 1) * chunk); ++i) {
    row_ptr[i] = (int32_t)run;
    run += counts[i];
  }
  if (t * chunk < nb && (t + 1) * chunk >= nb) row_ptr[nb] = (int32_t)run;  // the last non-empty chunk
  if (nb == 0 && t == 0) row_ptr[0] = 0;
}

// ---------------------------------------------------------- synthetic data
__global__ void fill_normal_kernel(uint16_t* __restrict__ out, int64_t n, uint64_t seed, uint64_t stream,
                                   double mean, double std) {
  const uint64_t key = splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ull));
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t hsh = splitmix64(key + ((uint64_t)i >> 1));
    double u1 = ((double)(hsh >> 40) + 1.0) * (1.0 / 16777216.0);
    double u2 = (double)(hsh & 0xFFFFFFull) * (1.0 / 16777216.0);
    double r = sqrt(-2.0 * log(u1));
    double ang = 6.283185307179586 * u2;
    double z = (i & 1) ? r * sin(ang) : r * cos(ang);
    out[i] = f2bf((float)(mean + std * z));
  }
}


// ------------------------------------------------------ block-list validation
// One thread per query block: row_ptr[0] == 0, row_ptr non-decreasing and
// within [0, nnz] (so no col_idx entry past the caller's nnz is ever read),
// every col_idx of the row in [0, n_blocks) and strictly ascending.
// Violations are OR-ed into *flags (1: row_ptr[0] != 0 or row_ptr[n_blocks]
// != nnz, 2: row_ptr decreasing or outside [0, nnz], 4: column out of range,
// 8: columns not strictly ascending).
__global__ void validate_blocks_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
                                       int32_t n_blocks, int64_t nnz, int32_t* flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_blocks) return;
  int bad = 0;
  if (i == 0 && row_ptr[0] != 0) bad |= 1;
  if (i == n_blocks - 1 && (int64_t)row_ptr[n_blocks] != nnz) bad |= 1;
  const int p0 = row_ptr[i], p1 = row_ptr[i + 1];
  if (p1 < p0 || p0 < 0 || (int64_t)p1 > nnz) bad |= 2;
  int prev = -1;
  for (int p = p0; p < p1 && !(bad & 2); ++p) {
    const int c = col_idx[p];
    if (c < 0 || c >= n_blocks) bad |= 4;
    if (c <= prev) bad |= 8;
    prev = c;
  }
  if (bad) atomicOr(flags, bad);
}
}  // namespace

cudaError_t launch_prologue(const uint16_t* x, int64_t x_tok, int64_t x_head, uint16_t* y, int64_t y_tok,
                            int64_t y_head, int32_t seq_len, int32_t head_count, const uint16_t* w, float eps,
                            const uint16_t* table, int32_t half, cudaStream_t s) {
  int64_t rows = (int64_t)seq_len * head_count;
  if (rows == 0) return cudaSuccess;
  // the register-pair kernel reads table entries 16 bytes at a time
  if (table == nullptr || (half % 4 == 0 && ((uintptr_t)table & 15) == 0)) {
    prologue_pairs_kernel<<<(unsigned)((rows + 15) / 16), 256, 0, s>>>(x, x_tok, x_head, y, y_tok, y_head, seq_len,
                                                                        head_count, w, eps, table,
                                                                        table ? half : 64);
    return cudaGetLastError();
  }
  prologue_kernel<<<(unsigned)((rows + 15) / 16), 256, 0, s>>>(x, x_tok, x_head, y, y_tok, y_head, seq_len,
                                                             head_count, w, eps, table, half);
  return cudaGetLastError();
}

cudaError_t launch_prologue_qk(const uint16_t* q, int64_t q_tok, int64_t q_head, uint16_t* qn, const uint16_t* k,
                               int64_t k_tok, int64_t k_head, uint16_t* kn, int64_t n_tok, int32_t seq_len,
                               int32_t head_count, const uint16_t* wq, const uint16_t* wk, float eps,
                               const uint16_t* table, int32_t half, int sm_count, cudaStream_t s) {
  if ((int64_t)seq_len * head_count == 0) return cudaSuccess;
  const bool fast = (table == nullptr || (half % 8 == 0 && ((uintptr_t)table & 15) == 0)) &&
                    !((uintptr_t)wq & 15) && !((uintptr_t)wk & 15);
  if (!fast) {  // any other half: the per-operand kernels
    cudaError_t e = launch_prologue(k, k_tok, k_head, kn, n_tok, 128, seq_len, head_count, wk, eps, table, half, s);
    if (e != cudaSuccess) return e;
    return launch_prologue(q, q_tok, q_head, qn, n_tok, 128, seq_len, head_count, wq, eps, table, half, s);
  }
  ProOperand o0{k, k_tok, k_head, kn, n_tok, 128, wk};
  ProOperand o1{q, q_tok, q_head, qn, n_tok, 128, wq};
  // 8 warps per CTA, two operands: enough warps for every SM, at most one
  // token per warp
  int64_t want = ((int64_t)seq_len * 2 + 7) / 8;
  // two heads in flight per thread (measured best of 1-4 at config 2:
  // 0.88 ms for 5.12 GB, 0.89 of the copy bandwidth), three 256-thread CTAs
  // resident per SM at 80 registers
  constexpr int kHeadsInFlight = 2;
  int64_t cap = (int64_t)sm_count * 3;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  prologue_qk_kernel<kHeadsInFlight><<<grid, 256, 0, s>>>(o0, o1, seq_len, head_count, eps, table,
                                                            table ? half : 0);
  return cudaGetLastError();
}

cudaError_t launch_rope_table(const int32_t* pos, int32_t seq_len, int3 dims, const float* d_inv, int32_t half,
                              uint16_t* table, cudaStream_t s) {
  int64_t n = (int64_t)seq_len * half;
  if (n == 0) return cudaSuccess;
  rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(pos, seq_len, dims, d_inv, half, table);
  return cudaGetLastError();
}

cudaError_t launch_rope_table_shared(const float* pos, int32_t seq_len, const float* d_inv, int32_t n,
                                     uint16_t* table, cudaStream_t s) {
  int64_t total = (int64_t)seq_len * 3 * n;
  if (total == 0) return cudaSuccess;
  rope_table_shared_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(pos, seq_len, d_inv, n, table);
  return cudaGetLastError();
}

cudaError_t launch_mask_build(const h3c_mask_spec& sp, int32_t* counts, int32_t* row_ptr, int32_t* col_idx,
                              int64_t capacity, int64_t* d_nnz, cudaStream_t s) {
  MaskDev m;
  m.seq_len = sp.seq_len; m.block = sp.block; m.prefix_len = sp.prefix_len;
  m.frames = sp.frames; m.height = sp.height; m.width = sp.width;
  m.cell_t = sp.cell_t; m.cell_h = sp.cell_h; m.cell_w = sp.cell_w;
  m.radius_t = sp.radius_t; m.radius_h = sp.radius_h; m.radius_w = sp.radius_w;
  m.n_random = sp.n_random; m.seed = sp.seed;
  m.nb = (sp.seq_len + sp.block - 1) / sp.block;
  m.npb = (sp.prefix_len + sp.block - 1) / sp.block;
  size_t smem = (size_t)((m.nb + 31) / 32) * 4;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  mask_rows_kernel<<<m.nb, 256, smem, s>>>(m, counts, nullptr, nullptr, 0, 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  scan_kernel<<<1, 1024, 0, s>>>(counts, m.nb, row_ptr, d_nnz);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  mask_rows_kernel<<<m.nb, 256, smem, s>>>(m, nullptr, row_ptr, col_idx, capacity, 1);
  return cudaGetLastError();
}

cudaError_t launch_validate_blocks(const int32_t* row_ptr, const int32_t* col_idx, int32_t n_blocks, int64_t nnz,
                                   int32_t* flags, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  validate_blocks_kernel<<<(n_blocks + 255) / 256, 256, 0, s>>>(row_ptr, col_idx, n_blocks, nnz, flags);
  return cudaGetLastError();
}

cudaError_t launch_fill_normal(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream, double mean, double std,
                               int sm_count, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  int64_t cap = (int64_t)sm_count * 16;
  fill_normal_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(out, n, seed, stream, mean, std);
  return cudaGetLastError();
}

}  // namespace h3
