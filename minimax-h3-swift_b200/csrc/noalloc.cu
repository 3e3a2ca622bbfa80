// h3c_attn_fwd_noalloc: the fused prologue + block-sparse attention for
// callers that cannot allocate device memory.
//
// Who needs it: callers for whom cudaMalloc is off limits -- a host process
// that has handed all device memory to its own pool at start-up (an
// inference server, or a Swift/MLX host whose framework owns the device
// heap) and forbids further allocations, and latency-critical loops where an
// allocation's cost or failure at call time is not acceptable.
// h3c_attn_fwd needs a context whose workspace is grown with cudaMalloc;
// this entry point needs neither a context nor an allocation.
//
// How: the normalised Q and K that the fused path stages between the
// prologue kernel and the attention kernel live in one file-scope device
// array, g_noalloc_scratch, of kNoAllocScratchBytes (32 MiB).  Every GPU
// that loads this library holds that array until the process exits.  The
// limit is 2 * ceil(S/128)*128 * head_count * 128 * 2 bytes <= 32 MiB, i.e.
// padded tokens x heads <= 65,536 (S = 4,096 with 16 heads, S = 8,192 with
// 8); larger calls are rejected with H3C_ERR_CAPACITY.
//
// Rules for callers:
//  * It runs on the calling thread's current device.  The first call on a
//    device looks up the array's device address with cudaGetSymbolAddress
//    (host code cannot use the array's name as a device pointer); make that
//    first call before any stream capture begins.
//  * All calls share the one array and it keeps the last call's contents.
//    Calls that overlap on the GPU (different streams, or different host
//    threads, without ordering between them) race on it.  Nothing in it has
//    to start at zero: every row a call reads is written by that call first
//    (padding rows past seq_len are never read; TMA fills them with zeros).
//  * A bounded device wait that gives up (H3C_ERR_TIMEOUT: the output of that
//    call is invalid) is recorded in a second file-scope device word,
//    g_noalloc_status, cleared at the start of every call;
//    h3c_attn_fwd_noalloc_status() reads and clears it.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
__device__ __align__(16) int32_t g_noalloc_status;

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
int32_t* g_status_addr[kMaxDevices] = {};

// Device addresses of the scratch array and the status word on the current
// device, looked up once per device with that device current.
cudaError_t resolve(int dev, void** scratch, int32_t** status) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev] || !g_status_addr[dev]) {
    void* a = nullptr;
    void* b = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&b, g_noalloc_status);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = a;
    g_status_addr[dev] = (int32_t*)b;
  }
  *scratch = g_scratch_addr[dev];
  *status = g_status_addr[dev];
  return cudaSuccess;
}

h3c_status report(char* err, size_t err_len, h3c_status st, const char* msg) {
  if (err && err_len) {
    std::snprintf(err, err_len, "%s", msg);
  }
  return st;
}

}  // namespace

extern "C" h3c_status h3c_attn_fwd_noalloc(const h3c_attn_args* args, void* stream, char* err, size_t err_len) {
  if (err && err_len) err[0] = '\0';
  if (!args) return report(err, err_len, H3C_ERR_INVALID_ARGUMENT, "h3c_attn_fwd_noalloc: null args");
  const h3c_attn_args& a = *args;
  if (!(a.flags & H3C_FUSE_PROLOGUE))
    return report(err, err_len, H3C_ERR_INVALID_ARGUMENT,
                  "h3c_attn_fwd_noalloc: only the fused path (H3C_FUSE_PROLOGUE) uses scratch; call h3c_attn_fwd");
  if (a.flags & H3C_KERNEL_MMA_SYNC)
    return report(err, err_len, H3C_ERR_UNSUPPORTED, "h3c_attn_fwd_noalloc: tcgen05 kernel only");
  {
    std::string msg;
    h3c_status st = h3::check_attn_args(args, "h3c_attn_fwd_noalloc", &msg);
    if (st != H3C_OK) return report(err, err_len, st, msg.c_str());
  }
  const bool rope = !(a.flags & H3C_NO_ROPE);

  const int n_blocks = (a.seq_len + 127) / 128;
  const size_t rows = (size_t)n_blocks * 128 * (size_t)a.head_count;
  const size_t need = 2 * rows * 128 * sizeof(uint16_t);
  if (need > kNoAllocScratchBytes) {
    char msg[200];
    std::snprintf(msg, sizeof(msg),
                  "h3c_attn_fwd_noalloc: needs %zu bytes of scratch, the fixed limit is %zu "
                  "(padded tokens x heads <= 65536); use h3c_attn_fwd",
                  need, kNoAllocScratchBytes);
    return report(err, err_len, H3C_ERR_CAPACITY, msg);
  }

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return report(err, err_len, H3C_ERR_NO_DEVICE, "h3c_attn_fwd_noalloc: no usable current device");
  void* scratch = nullptr;
  int32_t* status = nullptr;
  {
    cudaError_t e = resolve(dev, &scratch, &status);
    if (e != cudaSuccess) return report(err, err_len, H3C_ERR_CUDA, cudaGetErrorString(e));
  }

  cudaStream_t s = (cudaStream_t)stream;
  const int64_t ho = a.head_offset;
  h3::AttnLaunch L{};
  const uint16_t* q = (const uint16_t*)a.q.ptr + ho * a.q.head_stride;
  const uint16_t* k = (const uint16_t*)a.k.ptr + ho * a.k.head_stride;
  uint16_t* kn = (uint16_t*)scratch;
  uint16_t* qn = kn + rows * 128;
  const uint16_t* table = rope ? (const uint16_t*)a.rope_table : nullptr;
  const int half = rope ? a.rope_half : 0;
  const int64_t ntok = (int64_t)a.head_count * 128;
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  int sms = 148;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = h3::launch_prologue_qk(q, a.q.token_stride, a.q.head_stride, qn, k, a.k.token_stride, a.k.head_stride, kn,
                               ntok, a.seq_len, a.head_count, (const uint16_t*)a.q_norm_weight,
                               (const uint16_t*)a.k_norm_weight, a.eps, table, half, sms, s);
  if (e != cudaSuccess) return report(err, err_len, H3C_ERR_CUDA, cudaGetErrorString(e));
  L.q = qn; L.q_tok = ntok; L.q_head = 128;
  L.k = kn; L.k_tok = ntok; L.k_head = 128;
  L.v = (const uint16_t*)a.v.ptr + ho * a.v.head_stride; L.v_tok = a.v.token_stride; L.v_head = a.v.head_stride;
  L.o = (uint16_t*)a.out.ptr + ho * a.out.head_stride; L.o_tok = a.out.token_stride; L.o_head = a.out.head_stride;
  L.seq_len = a.seq_len;
  L.n_blocks = n_blocks;
  L.head_count = a.head_count;
  L.scale_log2 = a.scale * 1.4426950408889634f;
  L.row_ptr = a.row_ptr;
  L.col_idx = a.col_idx;
  L.status = status;
  L.wait_limit_ns = 4000000000ull;
  L.drop_item = -1;
  L.pdl = (a.flags & H3C_FUSE_PROLOGUE) ? 1 : 0;
  // the same host-side fault-injection hooks as h3c_attn_fwd (tests only)
  if (const char* d = getenv("H3C_TEST_DROP_ITEM")) L.drop_item = atoi(d);
  if (const char* w = getenv("H3C_TEST_WAIT_LIMIT_NS")) L.wait_limit_ns = strtoull(w, nullptr, 10);
  std::string why;
  e = h3::launch_attn_tc(L, s, &why);
  if (e != cudaSuccess) {
    why += cudaGetErrorString(e);
    return report(err, err_len, H3C_ERR_CUDA, why.c_str());
  }
  return H3C_OK;
}

extern "C" h3c_status h3c_attn_fwd_noalloc_status(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return H3C_ERR_NO_DEVICE;
  void* scratch = nullptr;
  int32_t* status = nullptr;
  if (resolve(dev, &scratch, &status) != cudaSuccess) return H3C_ERR_CUDA;
  int32_t word = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&word, status, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemset(status, 0, sizeof(int32_t)) != cudaSuccess)
    return H3C_ERR_CUDA;
  return (h3c_status)word;
}
