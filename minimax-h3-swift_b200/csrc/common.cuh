// Shared helpers of the H3 attention library (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "h3cuda.h"

struct h3c_ctx {
  int device = 0;
  std::string err;
  cudaDeviceProp prop{};
  void* workspace = nullptr;      // normalised keys/queries of the fused path
  size_t workspace_bytes = 0;
  cudaEvent_t workspace_done = nullptr;  // recorded after the last launch that read the workspace
  void* comm = nullptr;           // h3c_comm_state of the sequence-sharded path
  int64_t* d_counter = nullptr;   // small device scratch: [0] mask builder nnz, [1] kernel status word,
                                  // [2] block-list validation flags
};

namespace h3 {

constexpr int kHeadDim = 128;
constexpr int kBlock = 128;

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// round-to-nearest-even; identical to the CPU checker's conversion
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// Normalised K and Q of the fused call in one launch (falls back to two
// launch_prologue calls for a half that is not a multiple of 8); qn/kn rows
// are [seq, head_count, 128] with token stride n_tok.
cudaError_t launch_prologue_qk(const uint16_t* q, int64_t q_tok, int64_t q_head, uint16_t* qn, const uint16_t* k,
                               int64_t k_tok, int64_t k_head, uint16_t* kn, int64_t n_tok, int32_t seq_len,
                               int32_t head_count, const uint16_t* wq, const uint16_t* wk, float eps,
                               const uint16_t* table, int32_t half, int sm_count, cudaStream_t s);

}  // namespace h3

#define H3_CUDA_TRY(ctx, expr)                                                   \
  do {                                                                           \
    cudaError_t e_ = (expr);                                                     \
    if (e_ != cudaSuccess) {                                                     \
      if (ctx) (ctx)->err = std::string(#expr) + ": " + cudaGetErrorString(e_);  \
      return H3C_ERR_CUDA;                                                       \
    }                                                                            \
  } while (0)

// Launchers implemented in the kernel translation units.
namespace h3 {

struct AttnLaunch {
  // operands (bf16), element strides
  const uint16_t* q; int64_t q_tok, q_head;
  const uint16_t* k; int64_t k_tok, k_head;
  const uint16_t* v; int64_t v_tok, v_head;
  uint16_t* o; int64_t o_tok, o_head;
  int32_t seq_len, n_blocks, head_count;
  float scale_log2;               // scale * log2(e)
  const int32_t* row_ptr;
  const int32_t* col_idx;
  int32_t* status;                // device status word (bounded waits), may be null
  uint64_t wait_limit_ns;         // bound of every mbarrier wait
  int32_t drop_item;              // test hook: K/V ring item the producer skips (-1: none)
  int32_t pdl;                    // 1: launched as a programmatic dependent of the prologue kernel
                                  // just before it on the stream (q/k are its output)
};

// Argument checks shared by every attention entry point: H3C_OK, or a status
// with the reason in *msg (``who`` names the entry point in the message).
h3c_status check_attn_args(const h3c_attn_args* a, const char* who, std::string* msg);

cudaError_t launch_attn_mma(const AttnLaunch& a, cudaStream_t s);
cudaError_t launch_attn_tc(const AttnLaunch& a, cudaStream_t s, std::string* err);
cudaError_t launch_prologue(const uint16_t* x, int64_t x_tok, int64_t x_head, uint16_t* y, int64_t y_tok,
                            int64_t y_head, int32_t seq_len, int32_t head_count, const uint16_t* w,
                            float eps, const uint16_t* table, int32_t half, cudaStream_t s);

// Normalised K and Q of the fused call in one launch (falls back to two
// launch_prologue calls for a half that is not a multiple of 8); qn/kn rows
// are [seq, head_count, 128] with token stride n_tok.
cudaError_t launch_prologue_qk(const uint16_t* q, int64_t q_tok, int64_t q_head, uint16_t* qn, const uint16_t* k,
                               int64_t k_tok, int64_t k_head, uint16_t* kn, int64_t n_tok, int32_t seq_len,
                               int32_t head_count, const uint16_t* wq, const uint16_t* wk, float eps,
                               const uint16_t* table, int32_t half, int sm_count, cudaStream_t s);

}  // namespace h3
