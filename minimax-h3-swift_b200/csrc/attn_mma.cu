// Block-sparse attention forward on the legacy warp-level tensor path
// (mma.sync m16n8k16 bf16 -> fp32).  This is the bisection kernel: simple,
// obviously correct, and the baseline the tcgen05 kernel in attn_tc.cu has to
// beat.  Semantics follow the streaming recurrence of
// Sources/H3Attention/AxialReference.swift:116-171 over the kept key blocks of
// the compacted block list (ascending order), with key columns past seq_len
// masked.
//
// CTA = one 128-row query block of one head; 8 warps x 16 query rows.  Key and
// value tiles of 64 keys are double-buffered in shared memory with cp.async;
// shared rows are 256 B with the 16-byte chunk index XOR-swizzled by (row & 7)
// so that ldmatrix reads are bank-conflict free.
#include <mutex>

#include "common.cuh"

namespace h3 {
namespace {

constexpr int kRows = 128;      // query rows per CTA
constexpr int kTileKeys = 64;   // keys per pipeline stage
constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// byte offset of 16-byte chunk c of row r in a [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Load rows [r0, r0+nrows) x 128 of a strided bf16 operand into a swizzled
// tile; rows at or past seq_len are zero-filled.
__device__ __forceinline__ void load_tile(uint32_t sbase, const uint16_t* g, int64_t tok, int r0, int nrows,
                                          int seq_len) {
  for (int i = threadIdx.x; i < nrows * 16; i += kThreads) {
    int r = i >> 4, c = i & 15;
    int s = r0 + r;
    bool ok = s < seq_len;
    const uint16_t* src = g + (int64_t)(ok ? s : 0) * tok + c * 8;
    cp_async16(sbase + swz(r, c), src, ok);
  }
}

__global__ void __launch_bounds__(kThreads, 1) attn_mma_kernel(AttnLaunch a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                                  // 128 x 128
  uint8_t* sK = smem + kRows * 256;                    // 2 x 64 x 128
  uint8_t* sV = sK + 2 * kTileKeys * 256;              // 2 x 64 x 128

  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kRows;

  const uint16_t* gq = a.q + (int64_t)h * a.q_head;
  const uint16_t* gk = a.k + (int64_t)h * a.k_head;
  const uint16_t* gv = a.v + (int64_t)h * a.v_head;

  const int p0 = a.row_ptr[qb], p1 = a.row_ptr[qb + 1];
  const int ntiles = 2 * (p1 - p0);

  load_tile(smem_u32(sQ), gq, a.q_tok, q0, kRows, a.seq_len);
  cp_commit();
  auto issue = [&](int t) {
    int jb = a.col_idx[p0 + (t >> 1)];
    int k0 = jb * 128 + (t & 1) * kTileKeys;
    int st = t & 1;
    load_tile(smem_u32(sK + st * kTileKeys * 256), gk, a.k_tok, k0, kTileKeys, a.seq_len);
    load_tile(smem_u32(sV + st * kTileKeys * 256), gv, a.v_tok, k0, kTileKeys, a.seq_len);
  };
  if (ntiles > 0) issue(0);
  cp_commit();

  cp_wait<1>();
  __syncthreads();

  // Q fragments for this warp's 16 rows: 8 k-steps of 16 head dims.
  uint32_t qf[8][4];
  {
    const uint32_t base = smem_u32(sQ);
    int r = warp * 16 + (lane & 15);
    for (int kk = 0; kk < 8; ++kk) {
      int c = 2 * kk + (lane >> 4);
      ldsm_x4(base + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_lo = -1e30f, m_hi = -1e30f, l_lo = 0.f, l_hi = 0.f;

  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) issue(t + 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();

    const int st = t & 1;
    const uint32_t kb = smem_u32(sK + st * kTileKeys * 256);
    const uint32_t vb = smem_u32(sV + st * kTileKeys * 256);
    const int key0 = a.col_idx[p0 + (t >> 1)] * 128 + (t & 1) * kTileKeys;

    // S = Q K^T for 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles (16 keys)
        int key = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        int c = 2 * kk + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(key, c), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kk], b0, b1);
        mma16816(s[2 * np + 1], qf[kk], b2, b3);
      }
    }

    // online softmax in the log2 domain; invalid key columns -> -inf
    float mx_lo = -1e30f, mx_hi = -1e30f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      int col = key0 + n * 8 + 2 * (lane & 3);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int cc = col + (e & 1);
        float v = (cc < a.seq_len) ? s[n][e] * a.scale_log2 : -INFINITY;
        s[n][e] = v;
      }
      mx_lo = fmaxf(mx_lo, fmaxf(s[n][0], s[n][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(s[n][2], s[n][3]));
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffff, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffff, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffff, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffff, mx_hi, 2));
    float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    float r_lo = exp2f(m_lo - mn_lo), r_hi = exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float sum_lo = 0.f, sum_hi = 0.f;
    uint32_t pf[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float e0 = exp2f(s[n][0] - mn_lo), e1 = exp2f(s[n][1] - mn_lo);
      float e2 = exp2f(s[n][2] - mn_hi), e3 = exp2f(s[n][3] - mn_hi);
      sum_lo += e0 + e1;
      sum_hi += e2 + e3;
      pf[n >> 1][(n & 1) * 2 + 0] = pack_bf16(e0, e1);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_bf16(e2, e3);
    }
    l_lo = l_lo * r_lo + sum_lo;
    l_hi = l_hi * r_hi + sum_hi;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= r_lo;
      o[n][1] *= r_lo;
      o[n][2] *= r_hi;
      o[n][3] *= r_hi;
    }
    // O += P V : k = 64 keys (4 steps), n = 128 dims (16 tiles)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        int key = kk * 16 + (((lane >> 3) & 1) << 3) + (lane & 7);
        int c = 2 * np + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz(key, c), b0, b1, b2, b3);
        mma16816(o[2 * np], pf[kk], b0, b1);
        mma16816(o[2 * np + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();  // stage st is overwritten by the issue of tile t+2
  }

  // quad-reduce the row sums (each thread summed its own columns)
  l_lo += __shfl_xor_sync(0xffffffff, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffff, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffff, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffff, l_hi, 2);
  float inv_lo = 1.f / fmaxf(l_lo, 1e-30f), inv_hi = 1.f / fmaxf(l_hi, 1e-30f);
  int r_lo = q0 + warp * 16 + (lane >> 2), r_hi = r_lo + 8;
  uint16_t* go = a.o + (int64_t)h * a.o_head;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    int d = n * 8 + 2 * (lane & 3);
    if (r_lo < a.seq_len)
      *reinterpret_cast<uint32_t*>(go + (int64_t)r_lo * a.o_tok + d) = pack_bf16(o[n][0] * inv_lo, o[n][1] * inv_lo);
    if (r_hi < a.seq_len)
      *reinterpret_cast<uint32_t*>(go + (int64_t)r_hi * a.o_tok + d) = pack_bf16(o[n][2] * inv_hi, o[n][3] * inv_hi);
  }
}

}  // namespace

cudaError_t launch_attn_mma(const AttnLaunch& a, cudaStream_t s) {
  const int smem = kRows * 256 + 4 * kTileKeys * 256;
  // function attributes are per device context: set them once per device
  // (std::call_once: concurrent first calls from several host threads are safe)
  static std::once_flag once[64];
  static cudaError_t set_result[64];
  int dev = 0;
  cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [dev, smem] {
    set_result[dev] = cudaFuncSetAttribute(attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (set_result[dev] != cudaSuccess) return set_result[dev];
  dim3 grid(a.n_blocks, a.head_count);
  attn_mma_kernel<<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace h3
