// Block-sparse attention forward on the Blackwell tensor cores (sm_100a):
// tcgen05.mma with TMEM accumulators, TMA-staged K/V tiles, warp-specialised.
//
// Semantics: for every 128-row query block i and head h, one online softmax
// over the kept key blocks of row i of the compacted block list, in ascending
// order (Sources/H3Attention/AxialReference.swift:116-171 restated per block;
// key columns past seq_len are masked).  Output bf16, O / max(l, 1e-30).
//
// CTA = two adjacent query blocks (2i, 2i+1) of one head.  Their block lists
// overlap almost entirely (the local window of neighbouring blocks), so the
// CTA walks the union of the two lists and every K/V tile it loads serves
// both query tiles: half the L2->SM traffic of one query block per CTA.
// Roles:
//   warp 0      TMA producer: Q tiles once, then K and V of each union entry
//               into a 4-slot ring (two entries; an entry's K and V complete
//               one barrier), handing the entry's tile flags to the issuer
//   warp 1      MMA issuer (the whole warp, one lane elected per instruction):
//               S = Q K^T (SS), O += P V (TS),
//               in the order PV0 S0 PV1 S1 per entry so the two tiles'
//               softmax phases alternate; each PV starts once the softmax
//               has stored P for keys 0-95 (p_half) and waits for the last
//               32 keys (p_full) only before its last two steps
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax + epilogue of tile 0 (thread = query row = TMEM lane)
//   warps 8-11  softmax + epilogue of tile 1
// TMEM columns: tile t owns [256t, 256t+128) for S (P is written back over its
// first 64 columns as packed bf16) and [256t+128, 256t+256) for O.
// Shared tiles are 128 rows x 64 bf16 (128 B) boxes in the 128-byte swizzle;
// Q and K are K-major operands, V is an MN-major operand.
//
// Every mbarrier wait is bounded (wall-clock limit via %globaltimer).  On a
// timeout the waiting thread records H3C_ERR_TIMEOUT in the launch's status
// word and raises a CTA-wide abort flag; every role drains to the common
// exit, where TMEM is freed, and the waits of every other CTA see the status
// word and stop too.
#include <cuda.h>

#include <climits>
#include <mutex>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace h3 {
namespace {

constexpr int kThreads = 384;
constexpr int kStages = 4;
constexpr int kTileBytes = 128 * 128 * 2;   // one 128x128 bf16 tile
constexpr int kHalfBytes = kTileBytes / 2;  // one 128x64 swizzle box
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s

struct __align__(8) Barriers {
  uint64_t q_full[2];
  uint64_t kv_full[kStages];   // [0..1]: entry barriers (K and V of entry e on kv_full[e & 1])
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t p_half[2];   // P of the first 96 keys written (split hand-off)
  uint64_t o_full[2];
  uint32_t tmem_base;
  int32_t abort;
  // union entry e: bit 0 tile 0 active, bit 1 tile 1 active, bit 2 last
  // entry; written by the producer before the arrival on entry e's barrier,
  // read by the MMA issuer after waiting on it
  int32_t info[16];
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

constexpr int kSmemTiles = 2 * kTileBytes + kStages * kTileBytes;
constexpr int kSmemBytes = kSmemTiles + 1024 /*align slack*/ + 256 /*barriers*/;

// ------------------------------------------------------------- primitives
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false on abort/timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort_flag,
                                          int32_t* status, uint64_t limit_ns = kWaitLimitNs) {
  for (int i = 0; i < 64; ++i)
    if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    // another CTA's wait already gave up: stop instead of timing out again
    // (one status word per launch, so a systematic stall ends in one limit)
    if (status && *(volatile int32_t*)status != 0) {
      *abort_flag = 1;
      return false;
    }
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      if (status) atomicExch(status, (int32_t)H3C_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 3D tiled TMA load (no multicast): coordinates (d, token, head).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// The same three operations issued by a whole converged warp, one lane
// elected by elect.sync: the MMA warp runs its loop with all 32 lanes (no
// divergent single-lane branch around the issue), which measured 3% faster
// than a lane-0-only issuer (config 2 and dense).
__device__ __forceinline__ void mma_ss_w(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_ts_w(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tc_commit_w(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

#define H3_TMEM_LD16(addr, r)                                                                                 \
  asm volatile(                                                                                               \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];" \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),       \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])  \
      : "r"(addr))

#define H3_TMEM_ST16(addr, r)                                                                                  \
  asm volatile(                                                                                                \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" \
      ::"r"(addr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),       \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])              \
      : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for the share of the exponentials that would
// otherwise queue on the MUFU unit.  Cody-Waite split x = n + f with
// n = round(x) (via the 1.5*2^23 rounding constant) and f in [-0.5, 0.5];
// 2^f by a cubic fitted here for minimum relative error on that interval
// (max relative error 7.6e-5, far below the bf16 rounding P receives);
// 2^n is added to the exponent field.  x is clamped at -126 so that the
// result stays a non-negative finite number (masked entries give ~1e-38).
__device__ __forceinline__ float ex2_poly(float x) {
  constexpr float kC0 = 0.99992817640304565f, kC1 = 0.69326096773147583f, kC2 = 0.24260970950126648f,
                  kC3 = 0.055170975625514984f;
  constexpr float kRound = 12582912.0f;
  x = fmaxf(x, -126.0f);
  const float t = __fadd_rn(x, kRound);
  const float f = __fsub_rn(x, __fsub_rn(t, kRound));
  const float p = fmaf(fmaf(fmaf(kC3, f, kC2), f, kC1), f, kC0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (x0, x1) = (s0, s1) * k + b on the packed f32x2 pipe; k, b hold a scalar
// in both halves.
__device__ __forceinline__ void fma2(float& x0, float& x1, uint32_t s0, uint32_t s1, uint64_t k, uint64_t b) {
  asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%2, %3};\n\t"
      "fma.rn.ftz.f32x2 d, a, %4, %5;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(x0), "=f"(x1)
      : "r"(s0), "r"(s1), "l"(k), "l"(b));
}

__device__ __forceinline__ uint64_t add2(uint64_t acc, float a, float b) {
  uint64_t r;
  asm("{\n\t.reg .b64 t;\n\tmov.b64 t, {%2, %3};\n\tadd.rn.ftz.f32x2 %0, %1, t;\n\t}"
      : "=l"(r)
      : "l"(acc), "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ uint64_t dup2(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// descriptor version 1; lbo/sbo in bytes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128, N = 128.
constexpr uint32_t idesc_bf16(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((128u >> 3) << 17) |
         ((128u >> 4) << 24);
}

// ------------------------------------------------------------------ kernel
template <int EMU>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, AttnLaunch a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                        // 2 tiles
  uint8_t* sKV = smem + 2 * kTileBytes;      // kStages tiles
  Barriers* bars = (Barriers*)(smem + kSmemTiles);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile t = query block 2*blockIdx.x + t of head blockIdx.y
  const int qb0 = blockIdx.x * 2;
  const int h = blockIdx.y;
  const int ntile = (qb0 + 1 < a.n_blocks) ? 2 : 1;
  int tp0[2], tn[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    tp0[t] = t < ntile ? a.row_ptr[qb0 + t] : 0;
    tn[t] = t < ntile ? a.row_ptr[qb0 + t + 1] - tp0[t] : 0;
  }
  const int nkv = tn[0] + tn[1];
  volatile int32_t* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&bars->q_full[t]), 1);
      mbar_init(smem_u32(&bars->s_full[t]), 1);
      mbar_init(smem_u32(&bars->p_full[t]), 128);
      mbar_init(smem_u32(&bars->p_half[t]), 128);
      mbar_init(smem_u32(&bars->o_full[t]), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars->kv_full[s]), 1);
      mbar_init(smem_u32(&bars->kv_empty[s]), 1);
    }
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&bars->tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Register split: the launch gives 384 x 168; the producer/MMA warpgroup
  // keeps 72 and the two softmax warpgroups take 216 each
  // (4*32*72 + 8*32*216 = 64512 = 384*168; the host checks the launch count).
  // Neither side spills at this split.

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;");
   if (nkv > 0) {
    if (warp == 0) {
      // ------------------------------------------------------- TMA producer
      // Walks the union of the two tiles' ascending block lists; every key
      // block in the union is loaded once (K then V) and serves both tiles.
      if (lane == 0) {
        // q and k may be the output of the prologue kernel this grid was
        // launched as a dependent of: wait for it before the first load
        if (a.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int t = 0; t < ntile; ++t) {
          uint32_t bar = smem_u32(&bars->q_full[t]);
          mbar_expect_tx(bar, kTileBytes);
          uint32_t dst = smem_u32(sQ + t * kTileBytes);
          tma_load_3d(dst, &tm_q, bar, 0, (qb0 + t) * 128, h);
          tma_load_3d(dst + kHalfBytes, &tm_q, bar, 64, (qb0 + t) * 128, h);
        }
        // Union entry e: K into ring item 2e, V into item 2e+1, both on the
        // entry's barrier kv_full[e & 1] (one wait covers K and V).
        int issued = 0;  // entries whose loads were issued
        bool ok = true;
        auto load_entry = [&](int e, int jb, int info) {
          const int sk = (2 * e) % kStages, sv = (2 * e + 1) % kStages;
          const uint32_t phk = (uint32_t)(((2 * e) / kStages) & 1), phv = (uint32_t)(((2 * e + 1) / kStages) & 1);
          if (!mbar_wait(smem_u32(&bars->kv_empty[sk]), phk ^ 1u, abort_flag, a.status, a.wait_limit_ns) ||
              !mbar_wait(smem_u32(&bars->kv_empty[sv]), phv ^ 1u, abort_flag, a.status, a.wait_limit_ns)) {
            ok = false;
            return;
          }
          const uint32_t bar = smem_u32(&bars->kv_full[e & 1]);
          bars->info[e & 15] = info;
          mbar_expect_tx(bar, 2 * kTileBytes);
          // host-side fault injection for tests: a dropped item's load never
          // happens, so its entry never completes
          if (2 * e != a.drop_item) {
            const uint32_t dst = smem_u32(sKV + sk * kTileBytes);
            tma_load_3d(dst, &tm_k, bar, 0, jb * 128, h);
            tma_load_3d(dst + kHalfBytes, &tm_k, bar, 64, jb * 128, h);
          }
          if (2 * e + 1 != a.drop_item) {
            const uint32_t dst = smem_u32(sKV + sv * kTileBytes);
            tma_load_3d(dst, &tm_v, bar, 0, jb * 128, h);
            tma_load_3d(dst + kHalfBytes, &tm_v, bar, 64, jb * 128, h);
          }
          issued = e + 1;
        };
        int i0 = 0, i1 = 0;
        for (int e = 0; ok && (i0 < tn[0] || i1 < tn[1]); ++e) {
          const int c0 = i0 < tn[0] ? a.col_idx[tp0[0] + i0] : INT_MAX;
          const int c1 = i1 < tn[1] ? a.col_idx[tp0[1] + i1] : INT_MAX;
          const int u = min(c0, c1);
          i0 += (c0 == u);
          i1 += (c1 == u);
          const bool last = i0 >= tn[0] && i1 >= tn[1];
          load_entry(e, u, (c0 == u ? 1 : 0) | (c1 == u ? 2 : 0) | (last ? 4 : 0));
        }
        // Drain: wait for the last loads to land before anyone may exit.
        if (!ok) {
          for (int m = (issued > 2 ? issued - 2 : 0); m < issued; ++m) {
            volatile int32_t zero = 0;
            mbar_wait(smem_u32(&bars->kv_full[m & 1]), (uint32_t)((m >> 1) & 1), &zero, nullptr);
          }
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      // Union entry e owns ring items 2e (K) and 2e+1 (V).  Per entry, for
      // each tile in turn: the PV of the tile's previous entry (its P is ready
      // once the softmax arrives), then the tile's S for this entry, so the
      // tiles ping-pong between MMA and softmax and their exponentials (the
      // MUFU unit's load equals the tensor pipe's) rarely overlap.  K(e) is
      // released once the S of every tile active at e is issued; V(e) once
      // both tiles' PVs of e are issued (while entry e+1 is processed).
      {
        // lane 0 waits and broadcasts the outcome, so the warp stays converged
        auto iwait = [&](uint32_t bar, uint32_t par) -> bool {
          int r = 0;
          if (lane == 0) r = mbar_wait(bar, par, abort_flag, a.status, a.wait_limit_ns) ? 1 : 0;
          return __shfl_sync(0xffffffff, r, 0) != 0;
        };
        constexpr uint32_t kIdS = idesc_bf16(false);
        constexpr uint32_t kIdPV = idesc_bf16(true);
        bool ok = true;
        for (int t = 0; t < ntile && ok; ++t)
          ok = iwait(smem_u32(&bars->q_full[t]), 0);
        tc_fence_after();
        // Per-tile state lives in named scalars and every per-tile step is
        // instantiated for a compile-time tile index, so nothing here is
        // dynamically indexed (which would put it in local memory, on the
        // issue path).
        int pend0 = -1, pend1 = -1;  // union entry whose PV is still due, per tile
        int ns0 = 0, ns1 = 0;        // S issued per tile
        int landed = -1;  // last union entry whose K and V are known to have landed
        auto wait_entry = [&](int e) -> bool {
          if (e <= landed) return true;
          if (!iwait(smem_u32(&bars->kv_full[e & 1]), (uint32_t)((e >> 1) & 1)))
            return false;
          tc_fence_after();
          landed = e;
          return true;
        };
        auto issue_pv = [&](auto tile) -> bool {
          constexpr int t = decltype(tile)::value;
          int& pend = t == 0 ? pend0 : pend1;
          const int nst = t == 0 ? ns0 : ns1;
          const int other = t == 0 ? pend1 : pend0;
          const int e = pend;
          // split hand-off: the first six PV steps (keys 0-95) need only
          // p_half; p_full is awaited before the last two
          if (!iwait(smem_u32(&bars->p_half[t]), (uint32_t)((nst - 1) & 1)))
            return false;
          tc_fence_after();
          const int item = 2 * e + 1;
          if (!wait_entry(e)) return false;
          // descriptors are built once per tile; the start-address field
          // (bits 0-13, address >> 4) is advanced by plain addition (no
          // carry: shared addresses stay below 2^18)
          const uint64_t vdesc = smem_desc(smem_u32(sKV + (item % kStages) * kTileBytes), kHalfBytes, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            if (kk == 6) {
              if (!iwait(smem_u32(&bars->p_full[t]), (uint32_t)((nst - 1) & 1))) return false;
              tc_fence_after();
            }
            mma_ts_w(tmem + 256 * t + 128, tmem + 256 * t + kk * 8, vdesc + (uint64_t)((kk * 2048) >> 4),
                   kIdPV, (nst > 1 || kk > 0) ? 1u : 0u);
          }
          pend = -1;
          if (other != e) tc_commit_w(smem_u32(&bars->kv_empty[item % kStages]));
          return true;
        };
        auto issue_s = [&](auto tile, int e) {
          constexpr int t = decltype(tile)::value;
          const uint64_t qdesc = smem_desc(smem_u32(sQ + t * kTileBytes), 16, 1024);
          const uint64_t kdesc = smem_desc(smem_u32(sKV + ((2 * e) % kStages) * kTileBytes), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
            mma_ss_w(tmem + 256 * t, qdesc + (uint64_t)(off >> 4), kdesc + (uint64_t)(off >> 4), kIdS,
                   kk > 0 ? 1u : 0u);
          }
          tc_commit_w(smem_u32(&bars->s_full[t]));
          (t == 0 ? pend0 : pend1) = e;
          ++(t == 0 ? ns0 : ns1);
        };
        using T0 = std::integral_constant<int, 0>;
        using T1 = std::integral_constant<int, 1>;
        // The producer hands over each union entry's active tiles in shared
        // memory, so this thread issues no global loads.
        for (int e = 0; ok; ++e) {
          if (pend0 >= 0) ok = issue_pv(T0{});
          if (!ok || !wait_entry(e)) {
            ok = false;
            break;
          }
          const int info = ((volatile int32_t*)bars->info)[e & 15];
          if (info & 1) issue_s(T0{}, e);
          if (pend1 >= 0) ok = issue_pv(T1{});
          if (ok && (info & 2)) issue_s(T1{}, e);
          if (ok) tc_commit_w(smem_u32(&bars->kv_empty[(2 * e) % kStages]));
          if (info & 4) break;
        }
        if (ok && ntile > 0) {
          if (pend0 >= 0) ok = issue_pv(T0{});
          if (ok) tc_commit_w(smem_u32(&bars->o_full[0]));
        }
        if (ok && ntile > 1) {
          if (pend1 >= 0) ok = issue_pv(T1{});
          if (ok) tc_commit_w(smem_u32(&bars->o_full[1]));
        }
        // on an abort: every MMA issued so far retires before the exit
        // releases TMEM
        if (!ok)
          for (int t = 0; t < ntile; ++t) tc_commit_w(smem_u32(&bars->o_full[t]));
      }
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;");
    {
      // --------------------------------------------------- softmax + epilogue
      const int t = (warp - 4) >> 2;
      const int q = warp & 3;  // TMEM lane quarter this warp may access
      const int p0 = t ? tp0[1] : tp0[0];
      const int nkv = t ? tn[1] : tn[0];
      if (t < ntile && nkv == 0) {
        // a query block with no kept key block: O / max(l, 1e-30) with l = 0
        const int row = (qb0 + t) * 128 + 32 * q + lane;
        if (row < a.seq_len) {
          uint4* go = reinterpret_cast<uint4*>(a.o + (int64_t)h * a.o_head + (int64_t)row * a.o_tok);
#pragma unroll
          for (int c = 0; c < 16; ++c) go[c] = make_uint4(0, 0, 0, 0);
        }
      }
      if (t < ntile && nkv > 0) {
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t tS = tmem + lane_base + 256 * t;
        const uint32_t tO = tS + 128;
        const float sl2 = a.scale_log2;
        float m = -1e30f, l = 0.f;
        bool ok = true;
        // only the sequence's last block can be partial, and it can only be
        // the last kept block of this row (the list is ascending)
        const int last_valid = a.seq_len - a.col_idx[p0 + nkv - 1] * 128;
        const uint64_t sl2x2 = dup2(sl2);
        for (int j = 0; j < nkv; ++j) {
          if (!mbar_wait(smem_u32(&bars->s_full[t]), (uint32_t)(j & 1), abort_flag, a.status, a.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t s[128];
#pragma unroll
          for (int c = 0; c < 8; ++c) H3_TMEM_LD16(tS + 16 * c, (&s[16 * c]));
          tmem_wait_ld();
          const int valid = (j == nkv - 1) ? last_valid : 128;
          if (valid < 128) {
#pragma unroll
            for (int c = 0; c < 128; ++c)
              if (c >= valid) s[c] = __float_as_uint(-INFINITY);
          }
          // row max: 8 independent chains of 16 (short dependency chains)
          float mxa[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float r = __uint_as_float(s[16 * g]);
#pragma unroll
            for (int c = 1; c < 15; c += 2)
              r = max3(r, __uint_as_float(s[16 * g + c]), __uint_as_float(s[16 * g + c + 1]));
            mxa[g] = fmaxf(r, __uint_as_float(s[16 * g + 15]));
          }
          const float mx = max3(max3(mxa[0], mxa[1], mxa[2]), max3(mxa[3], mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7]));
          const float mxs = mx * sl2;
          // Lazy rescale: keep the running max unless the new one exceeds it
          // by more than 8 (a factor 256 in the exponentials).
          bool need = (j == 0) ? false : (mxs > m + 8.0f);
          if (j == 0) m = mxs;
          if (__any_sync(0xffffffff, need)) {
            const float f = need ? ex2(m - mxs) : 1.0f;
            if (need) {
              l *= f;
              m = mxs;
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t o[16];
              H3_TMEM_LD16(tO + 16 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
              H3_TMEM_ST16(tO + 16 * c, o);
            }
          }
          const uint64_t negm = dup2(-m);
          uint64_t sum2 = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float x0, x1;
              fma2(x0, x1, s[32 * c + 2 * e], s[32 * c + 2 * e + 1], sl2x2, negm);
              float p0v, p1v;
              if ((e & 7) < EMU) {
                p0v = ex2_poly(x0);
                p1v = ex2_poly(x1);
              } else {
                p0v = ex2(x0);
                p1v = ex2(x1);
              }
              sum2 = add2(sum2, p0v, p1v);
              pk[e] = pack_bf16(p0v, p1v);
            }
            H3_TMEM_ST16(tS + 16 * c, pk);
            if (c == 2) {  // keys 0-95 of P are in TMEM: the first six PV steps may start
              tmem_wait_st();
              tc_fence_before();
              mbar_arrive(smem_u32(&bars->p_half[t]));
            }
          }
          l += __uint_as_float((uint32_t)sum2) + __uint_as_float((uint32_t)(sum2 >> 32));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&bars->p_full[t]));
        }
        if (ok && mbar_wait(smem_u32(&bars->o_full[t]), 0, abort_flag, a.status, a.wait_limit_ns)) {
          tc_fence_after();
          const int row = (qb0 + t) * 128 + 32 * q + lane;
          const float inv = 1.0f / fmaxf(l, 1e-30f);
          uint16_t* go = a.o + (int64_t)h * a.o_head + (int64_t)row * a.o_tok;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            H3_TMEM_LD16(tO + 16 * c, o);
            tmem_wait_ld();
            uint4 w0, w1;
            w0.x = pack_bf16(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv);
            w0.y = pack_bf16(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv);
            w0.z = pack_bf16(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv);
            w0.w = pack_bf16(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv);
            w1.x = pack_bf16(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv);
            w1.y = pack_bf16(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv);
            w1.z = pack_bf16(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv);
            w1.w = pack_bf16(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv);
            if (row < a.seq_len) {
              reinterpret_cast<uint4*>(go + 16 * c)[0] = w0;
              reinterpret_cast<uint4*>(go + 16 * c)[1] = w1;
            }
          }
        }
      }
    }
  }

  // ------------------------------------------------------------------ exit
  tc_fence_before();
  __syncthreads();
  if (bars->abort) {
    // every issuer committed its MMAs to o_full[t], aborted or not; wait
    // (bounded) for them so that no MMA is still writing TMEM when it is
    // released
    volatile int32_t zero = 0;
    if (warp == 2)
      for (int t = 0; t < ntile; ++t) mbar_wait(smem_u32(&bars->o_full[t]), 0, &zero, nullptr);
    __syncwarp();
  }
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// --------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Looked up once per process (thread-safe static initialisation).
EncodeTiledFn get_encode() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (EncodeTiledFn)p;
    return (EncodeTiledFn) nullptr;
  }();
  return fn;
}

// (d, token, head) view of a strided bf16 operand, boxes of 64 x 128 x 1.
bool make_map(CUtensorMap* m, const void* base, int64_t tok_stride, int64_t head_stride, int seq, int heads,
              std::string* err) {
  EncodeTiledFn enc = get_encode();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable; ";
    return false;
  }
  cuuint64_t dims[3] = {128, (cuuint64_t)seq, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)tok_stride * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + "); ";
    return false;
  }
  return true;
}

constexpr int kDefaultEmu = 0;

template <int EMU>
cudaError_t launch_variant(dim3 grid, cudaStream_t s, const CUtensorMap& mq, const CUtensorMap& mk,
                           const CUtensorMap& mv, const AttnLaunch& a) {
  // function attributes are per device context: set them once per device
  // (std::call_once: host threads making their first call together are safe)
  static std::once_flag once[64];  // one table per template instance
  static cudaError_t set_result[64];
  int dev = 0;
  cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [dev] {
    cudaError_t e =
        cudaFuncSetAttribute(attn_tc_kernel<EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    // setmaxnreg draws on the registers the block was launched with; the
    // kernel's split needs exactly 168 per thread at launch.
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, attn_tc_kernel<EMU>);
    if (e == cudaSuccess && fa.numRegs != 168) e = cudaErrorInvalidConfiguration;
    set_result[dev] = e;
  });
  if (set_result[dev] != cudaSuccess) return set_result[dev];
  // Programmatic dependent launch after the prologue: the CTAs are placed as
  // the prologue's retire and do their set-up (barriers, TMEM) while its
  // tail runs; the producer waits for the prologue before loading Q and K.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_tc_kernel<EMU>, mq, mk, mv, a);
}

}  // namespace

cudaError_t launch_attn_tc(const AttnLaunch& a, cudaStream_t s, std::string* err) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a.q, a.q_tok, a.q_head, a.seq_len, a.head_count, err) ||
      !make_map(&mk, a.k, a.k_tok, a.k_head, a.seq_len, a.head_count, err) ||
      !make_map(&mv, a.v, a.v_tok, a.v_head, a.seq_len, a.head_count, err))
    return cudaErrorInvalidValue;
  // Share of exponentials computed on the FMA pipe, in eighths (tuning knob
  // H3C_EXP_EMU, read once; default chosen by measurement).
  static const int emu = [] {
    const char* env = getenv("H3C_EXP_EMU");
    const int v = env ? atoi(env) : kDefaultEmu;
    return (v < 0 || v > 8) ? kDefaultEmu : v;
  }();
  dim3 grid((a.n_blocks + 1) / 2, a.head_count);
  switch (emu) {
    case 0: return launch_variant<0>(grid, s, mq, mk, mv, a);
    case 2: return launch_variant<2>(grid, s, mq, mk, mv, a);
    case 4: return launch_variant<4>(grid, s, mq, mk, mv, a);
    default: return launch_variant<kDefaultEmu>(grid, s, mq, mk, mv, a);
  }
}

}  // namespace h3
