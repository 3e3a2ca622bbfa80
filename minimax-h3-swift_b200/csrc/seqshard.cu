// Sequence-sharded attention over NCCL (one process per GPU).
//
// Each rank holds a contiguous, block-aligned slice of the tokens for every
// head: [S_r, H, D] with S_r = ceil(ceil(S / P) / 128) * 128.  One grouped
// send/recv all-to-all per operand turns that into [P * S_r, H / P, D] (every
// token, this rank's heads), the fused call runs on it, and one all-to-all
// returns the output slice.  The reference is single-process
// (FRAGILE_CONTRACTS.md: batch-1, one device), so this layout is new; it is
// the C-ABI counterpart of h3attention/sharding.py for callers that drive
// their own ranks (e.g. Swift).
//
// NCCL is opened with dlopen when a communicator is first created, reusing a
// libnccl.so.2 that the process has already loaded (for example PyTorch's),
// so the library has no link-time NCCL dependency.
//
// Failure detection: the communicator is created non-blocking when the NCCL
// in the process supports it (ncclCommInitRankConfig, 2.14+), and
// h3c_comm_wait bounds every wait on the exchange: it polls the stream and
// ncclCommGetAsyncError against a deadline and, when a peer never arrives,
// aborts the communicator (ncclCommAbort stops its kernels) and returns
// H3C_ERR_TIMEOUT instead of hanging -- the kernel-level counterpart of the
// reference's render cancellation (Sources/MiniMaxH3/RenderEngine.swift:
// 574-590).
#include <dlfcn.h>
#include <time.h>

#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

// The few NCCL entry points used, with the ABI of nccl.h (2.x).
typedef int ncclResult_t_;
typedef void* ncclComm_t_;
typedef struct {
  char internal[128];
} ncclUniqueId_;
enum { kNcclBfloat16 = 9 };  // ncclBfloat16
constexpr int kNcclSuccess = 0, kNcclInProgress = 7;

// ncclConfig_t as nccl.h 2.28 lays it out (fields are only ever appended;
// `size` and `version` tell the library how many of them it was given).
struct NcclConfig {
  size_t size;
  unsigned int magic;
  unsigned int version;
  int blocking, cgaClusterSize, minCTAs, maxCTAs;
  const char* netName;
  int splitShare, trafficClass;
  const char* commName;
  int collnetEnable, CTAPolicy, shrinkShare, nvlsCTAs, nChannelsPerNetPeer, nvlinkCentricSched;
};

NcclConfig nonblocking_config(int runtime_version) {
  NcclConfig c;
  c.size = sizeof(NcclConfig);
  c.magic = 0xcafebeef;
  // the struct above is 2.28's; an older library reads the prefix it knows
  c.version = (unsigned)(runtime_version < 22809 ? runtime_version : 22809);
  c.blocking = 0;
  c.cgaClusterSize = c.minCTAs = c.maxCTAs = INT_MIN;  // NCCL_CONFIG_UNDEF_INT
  c.netName = nullptr;
  c.splitShare = c.trafficClass = INT_MIN;
  c.commName = nullptr;
  c.collnetEnable = c.CTAPolicy = c.shrinkShare = c.nvlsCTAs = c.nChannelsPerNetPeer = c.nvlinkCentricSched = INT_MIN;
  return c;
}

struct Nccl {
  ncclResult_t_ (*GetUniqueId)(ncclUniqueId_*);
  ncclResult_t_ (*CommInitRank)(ncclComm_t_*, int, ncclUniqueId_, int);
  ncclResult_t_ (*CommDestroy)(ncclComm_t_);
  ncclResult_t_ (*GroupStart)();
  ncclResult_t_ (*GroupEnd)();
  ncclResult_t_ (*Send)(const void*, size_t, int, int, ncclComm_t_, cudaStream_t);
  ncclResult_t_ (*Recv)(void*, size_t, int, int, ncclComm_t_, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t_);
  // optional (non-blocking communicators, bounded waits)
  ncclResult_t_ (*CommInitRankConfig)(ncclComm_t_*, int, ncclUniqueId_, int, NcclConfig*) = nullptr;
  ncclResult_t_ (*CommGetAsyncError)(ncclComm_t_, ncclResult_t_*) = nullptr;
  ncclResult_t_ (*CommAbort)(ncclComm_t_) = nullptr;
  ncclResult_t_ (*CommFinalize)(ncclComm_t_) = nullptr;
  ncclResult_t_ (*GetVersion)(int*) = nullptr;
  bool ok = false;
};

Nccl* nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    n.GetUniqueId = (decltype(n.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    n.CommInitRank = (decltype(n.CommInitRank))dlsym(h, "ncclCommInitRank");
    n.CommDestroy = (decltype(n.CommDestroy))dlsym(h, "ncclCommDestroy");
    n.GroupStart = (decltype(n.GroupStart))dlsym(h, "ncclGroupStart");
    n.GroupEnd = (decltype(n.GroupEnd))dlsym(h, "ncclGroupEnd");
    n.Send = (decltype(n.Send))dlsym(h, "ncclSend");
    n.Recv = (decltype(n.Recv))dlsym(h, "ncclRecv");
    n.GetErrorString = (decltype(n.GetErrorString))dlsym(h, "ncclGetErrorString");
    n.CommInitRankConfig = (decltype(n.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
    n.CommGetAsyncError = (decltype(n.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
    n.CommAbort = (decltype(n.CommAbort))dlsym(h, "ncclCommAbort");
    n.CommFinalize = (decltype(n.CommFinalize))dlsym(h, "ncclCommFinalize");
    n.GetVersion = (decltype(n.GetVersion))dlsym(h, "ncclGetVersion");
    n.ok = n.GetUniqueId && n.CommInitRank && n.CommDestroy && n.GroupStart && n.GroupEnd && n.Send && n.Recv &&
           n.GetErrorString;
  });
  return n.ok ? &n : nullptr;
}

h3c_status fail(h3c_ctx* ctx, h3c_status st, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return st;
}

// A call on a non-blocking communicator may return ncclInProgress: the
// operation is being set up in the background and counts as issued.
bool issued(ncclResult_t_ r) { return r == kNcclSuccess || r == kNcclInProgress; }

double now_ms() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return t.tv_sec * 1e3 + t.tv_nsec * 1e-6;
}

void nap() {
  timespec t{0, 100000};  // 100 us between polls
  nanosleep(&t, nullptr);
}

// One head chunk of the exchange: heads [h0, h0 + hc) of every rank's group
// of hp heads.  [S_r, H, D] strided view <-> [P][S_r][hc][D] contiguous,
// 16-byte vectors.  dir 0: view -> packed (before sending); dir 1: packed ->
// view (after receiving).
__global__ void pack_kernel(uint16_t* __restrict__ view, int64_t tok, int64_t head, uint16_t* __restrict__ packed,
                            int32_t s_r, int32_t P, int32_t hp, int32_t h0, int32_t hc, int dir) {
  const int64_t n = (int64_t)s_r * P * hc * 16;  // 16-byte chunks
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i & 15);
    int64_t r = i >> 4;
    const int hl = (int)(r % hc);
    r /= hc;
    const int64_t s = r % s_r;
    const int p = (int)(r / s_r);
    const int h = p * hp + h0 + hl;
    uint4* a = reinterpret_cast<uint4*>(view + s * tok + (int64_t)h * head) + c;
    uint4* b = reinterpret_cast<uint4*>(packed + (((int64_t)p * s_r + s) * hc + hl) * 128) + c;
    if (dir == 0) *b = *a;
    else *a = *b;
  }
}

}  // namespace

constexpr int kMaxChunks = 8;
constexpr int kDefaultChunks = 1;

struct h3c_comm_state {
  ncclComm_t_ comm = nullptr;
  bool nonblocking = false;
  bool aborted = false;  // after a timeout: the communicator is gone, init again
  int nranks = 0, rank = 0;
  void* buf = nullptr;
  size_t buf_bytes = 0;
  // the exchange stream and the events that chain it with the caller's
  // stream, created with the communicator
  cudaStream_t side = nullptr;
  cudaEvent_t start = nullptr, in_done[kMaxChunks] = {}, attn_done[kMaxChunks] = {}, out_done = nullptr;
};

namespace {
h3c_comm_state* comm_of(h3c_ctx* ctx) { return reinterpret_cast<h3c_comm_state*>(ctx->comm); }
}  // namespace

extern "C" {

h3c_status h3c_comm_unique_id(h3c_comm_id* out) {
  if (!out) return H3C_ERR_INVALID_ARGUMENT;
  Nccl* n = nccl();
  if (!n) return H3C_ERR_NCCL;
  ncclUniqueId_ id;
  if (n->GetUniqueId(&id) != 0) return H3C_ERR_NCCL;
  static_assert(sizeof(id) == sizeof(out->internal), "unique id size");
  std::memcpy(out->internal, id.internal, sizeof(id.internal));
  return H3C_OK;
}

h3c_status h3c_comm_init(h3c_ctx* ctx, const h3c_comm_id* id, int nranks, int rank) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!id || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_comm_init: bad id/nranks/rank");
  if (ctx->comm) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_comm_init: communicator already initialised");
  Nccl* n = nccl();
  if (!n) return fail(ctx, H3C_ERR_NCCL, "h3c_comm_init: libnccl.so.2 could not be loaded");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId_ uid;
  std::memcpy(uid.internal, id->internal, sizeof(uid.internal));
  auto* st = new h3c_comm_state();
  ncclResult_t_ r;
  int ver = 0;
  // H3C_NCCL_BLOCKING=1 keeps a blocking communicator (no abort on timeout)
  const char* blk = getenv("H3C_NCCL_BLOCKING");
  const bool want_blocking = blk && atoi(blk) != 0;
  if (!want_blocking && n->CommInitRankConfig && n->CommGetAsyncError && n->CommAbort && n->GetVersion &&
      n->GetVersion(&ver) == 0 && ver >= 21400) {
    NcclConfig cfg = nonblocking_config(ver);
    r = n->CommInitRankConfig(&st->comm, nranks, uid, rank, &cfg);
    st->nonblocking = true;
    // a non-blocking init completes in the background: wait for it, bounded
    const char* e = getenv("H3C_NCCL_INIT_TIMEOUT_MS");
    const double limit = e ? atof(e) : 300000.0;
    const double t0 = now_ms();
    while (r == kNcclInProgress && st->comm) {
      ncclResult_t_ a = kNcclInProgress;
      n->CommGetAsyncError(st->comm, &a);
      r = a;
      if (r != kNcclInProgress) break;
      if (now_ms() - t0 > limit) {
        n->CommAbort(st->comm);
        delete st;
        return fail(ctx, H3C_ERR_TIMEOUT, "h3c_comm_init: the other ranks did not join in time (communicator aborted)");
      }
      nap();
    }
  } else {
    r = n->CommInitRank(&st->comm, nranks, uid, rank);
  }
  if (r != 0) {
    if (st->comm && st->nonblocking) n->CommAbort(st->comm);
    delete st;
    return fail(ctx, H3C_ERR_NCCL, std::string("ncclCommInitRank: ") + n->GetErrorString(r));
  }
  st->nranks = nranks;
  st->rank = rank;
  ctx->comm = st;
  cudaError_t ce = cudaStreamCreateWithFlags(&st->side, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&st->start, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&st->out_done, cudaEventDisableTiming);
  for (int c = 0; c < kMaxChunks && ce == cudaSuccess; ++c) {
    ce = cudaEventCreateWithFlags(&st->in_done[c], cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&st->attn_done[c], cudaEventDisableTiming);
  }
  if (ce != cudaSuccess) {
    h3c_comm_destroy(ctx);
    return fail(ctx, H3C_ERR_CUDA, std::string("h3c_comm_init: stream/event creation: ") + cudaGetErrorString(ce));
  }
  return H3C_OK;
}

h3c_status h3c_comm_destroy(h3c_ctx* ctx) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  h3c_comm_state* st = comm_of(ctx);
  if (!st) return H3C_OK;
  cudaSetDevice(ctx->device);
  if (st->buf) cudaFree(st->buf);
  if (st->side) {
    cudaStreamSynchronize(st->side);
    cudaStreamDestroy(st->side);
  }
  for (cudaEvent_t e : {st->start, st->out_done})
    if (e) cudaEventDestroy(e);
  for (int c = 0; c < kMaxChunks; ++c) {
    if (st->in_done[c]) cudaEventDestroy(st->in_done[c]);
    if (st->attn_done[c]) cudaEventDestroy(st->attn_done[c]);
  }
  Nccl* n = nccl();
  if (n && st->comm && !st->aborted) {
    bool done = true;
    if (st->nonblocking && n->CommFinalize) {
      // a non-blocking communicator finalises in the background (bounded);
      // one that does not finish is aborted instead of destroyed
      ncclResult_t_ r = n->CommFinalize(st->comm);
      const double t0 = now_ms();
      while (r == kNcclInProgress && now_ms() - t0 < 30000.0) {
        nap();
        n->CommGetAsyncError(st->comm, &r);
      }
      done = r == kNcclSuccess;
    }
    if (done) n->CommDestroy(st->comm);
    else n->CommAbort(st->comm);
  }
  delete st;
  ctx->comm = nullptr;
  return H3C_OK;
}

h3c_status h3c_attn_fwd_seqshard(h3c_ctx* ctx, const h3c_attn_args* args, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  h3c_comm_state* st = comm_of(ctx);
  if (!st) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_attn_fwd_seqshard: call h3c_comm_init first");
  if (!args) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_attn_fwd_seqshard: null args");
  const h3c_attn_args& a = *args;
  const int P = st->nranks;
  if (a.head_dim != 128 || a.block != 128) return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_attn_fwd_seqshard: head_dim/block");
  if (a.heads <= 0 || a.heads % P || a.head_offset != 0 || a.head_count != a.heads)
    return fail(ctx, H3C_ERR_UNSUPPORTED,
                "h3c_attn_fwd_seqshard: all heads (head_offset 0, head_count == heads), heads divisible by ranks");
  if (a.seq_len <= 0) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_attn_fwd_seqshard: seq_len");
  const h3c_view* vs[4] = {&a.q, &a.k, &a.v, &a.out};
  for (const h3c_view* v : vs)
    if (!v->ptr || ((uintptr_t)v->ptr & 15) || v->token_stride <= 0 || v->head_stride <= 0 || (v->token_stride & 7) ||
        (v->head_stride & 7))
      return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_attn_fwd_seqshard: q/k/v/out need 16-byte aligned rows");
  Nccl* n = nccl();
  if (!n) return fail(ctx, H3C_ERR_NCCL, "h3c_attn_fwd_seqshard: NCCL unavailable");
  if (st->aborted)
    return fail(ctx, H3C_ERR_NCCL, "h3c_attn_fwd_seqshard: the communicator was aborted; h3c_comm_destroy and init again");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = (cudaStream_t)stream;

  // shard length: whole 128-token blocks, equal on every rank
  const int per = (a.seq_len + P - 1) / P;
  const int s_r = (per + 127) / 128 * 128;
  const int hp = a.heads / P;
  const size_t elems = (size_t)s_r * a.heads * 128;  // one operand slice == one exchanged operand
  const size_t need = 5 * elems * sizeof(uint16_t);  // send buffer + exchanged q, k, v and the output
  if (st->buf_bytes < need) {
    if (st->buf) {
      // the previous call (on any stream) ends with out_done on the side
      // stream, after every launch that used the buffer
      H3_CUDA_TRY(ctx, cudaEventSynchronize(st->out_done));
      H3_CUDA_TRY(ctx, cudaStreamSynchronize(st->side));
      cudaFree(st->buf);
      st->buf = nullptr;
      st->buf_bytes = 0;
    }
    H3_CUDA_TRY(ctx, cudaMalloc(&st->buf, need));
    st->buf_bytes = need;
  }
  // layout: [send | q_x | k_x | v_x | o_x]; each is split into head chunks
  // (chunk c holds heads [h0, h0 + hc) of every rank's group, all tokens);
  // o_x comes back through the chunk's part of send.
  uint16_t* send = (uint16_t*)st->buf;
  uint16_t* qx = send + elems;
  uint16_t* kx = qx + elems;
  uint16_t* vx = kx + elems;
  uint16_t* ox = vx + elems;
  const int threads = 256;
  const int blocks = ctx->prop.multiProcessorCount * 8;
  // Pipeline over head chunks: the exchange of chunk c+1 (side stream)
  // overlaps the attention of chunk c (caller's stream), and the output of
  // chunk c travels back while chunk c+1 computes.
  // H3C_SEQ_CHUNKS: head chunks of the pipeline (tuning knob), read once
  // (thread-safe static initialisation)
  static const int chunks_env = [] {
    const char* e = getenv("H3C_SEQ_CHUNKS");
    const int c = e ? atoi(e) : kDefaultChunks;
    return (c < 1 || c > kMaxChunks) ? kDefaultChunks : c;
  }();
  const int nchunk = hp < chunks_env ? hp : chunks_env;
  cudaStream_t x = st->side;

  auto exchange = [&](uint16_t* src, uint16_t* dst, size_t per_peer) -> h3c_status {
    if (!issued(n->GroupStart())) return fail(ctx, H3C_ERR_NCCL, "ncclGroupStart");
    for (int p = 0; p < P; ++p) {
      if (!issued(n->Send(src + p * per_peer, per_peer, kNcclBfloat16, p, st->comm, x)) ||
          !issued(n->Recv(dst + p * per_peer, per_peer, kNcclBfloat16, p, st->comm, x))) {
        n->GroupEnd();
        ncclResult_t_ a = kNcclSuccess;
        if (st->nonblocking) n->CommGetAsyncError(st->comm, &a);
        return fail(ctx, H3C_ERR_NCCL, std::string("ncclSend/ncclRecv (communicator state: ") + n->GetErrorString(a) + ")");
      }
    }
    ncclResult_t_ r = n->GroupEnd();
    if (!issued(r)) return fail(ctx, H3C_ERR_NCCL, std::string("ncclGroupEnd: ") + n->GetErrorString(r));
    if (r == kNcclInProgress) {
      // a non-blocking communicator launches the group in the background;
      // it must settle before the next NCCL call on it (bounded)
      const double t0 = now_ms();
      while (r == kNcclInProgress) {
        n->CommGetAsyncError(st->comm, &r);
        if (r == kNcclInProgress && now_ms() - t0 > 60000.0) {
          n->CommAbort(st->comm);
          st->aborted = true;
          return fail(ctx, H3C_ERR_TIMEOUT, "h3c_attn_fwd_seqshard: the exchange could not be launched (aborted)");
        }
      }
      if (r != kNcclSuccess) return fail(ctx, H3C_ERR_NCCL, std::string("ncclGroupEnd: ") + n->GetErrorString(r));
    }
    return H3C_OK;
  };
  auto chunk_of = [&](int c, int* h0, int* hc) {
    *h0 = c * hp / nchunk;
    *hc = (c + 1) * hp / nchunk - *h0;
  };
  auto send_out = [&](int c) -> h3c_status {
    int h0, hc;
    chunk_of(c, &h0, &hc);
    const size_t off = (size_t)P * s_r * h0 * 128, per_peer = (size_t)s_r * hc * 128;
    H3_CUDA_TRY(ctx, cudaStreamWaitEvent(x, st->attn_done[c], 0));
    h3c_status e = exchange(ox + off, send + off, per_peer);
    if (e != H3C_OK) return e;
    pack_kernel<<<blocks, threads, 0, x>>>((uint16_t*)a.out.ptr, a.out.token_stride, a.out.head_stride, send + off,
                                           s_r, P, hp, h0, hc, 1);
    H3_CUDA_TRY(ctx, cudaGetLastError());
    return H3C_OK;
  };

  H3_CUDA_TRY(ctx, cudaEventRecord(st->start, s));
  H3_CUDA_TRY(ctx, cudaStreamWaitEvent(x, st->start, 0));
  const h3c_view ins[3] = {a.q, a.k, a.v};
  uint16_t* outs[3] = {qx, kx, vx};
  for (int c = 0; c < nchunk; ++c) {
    int h0, hc;
    chunk_of(c, &h0, &hc);
    const size_t off = (size_t)P * s_r * h0 * 128, per_peer = (size_t)s_r * hc * 128;
    for (int i = 0; i < 3; ++i) {
      pack_kernel<<<blocks, threads, 0, x>>>((uint16_t*)ins[i].ptr, ins[i].token_stride, ins[i].head_stride,
                                             send + off, s_r, P, hp, h0, hc, 0);
      H3_CUDA_TRY(ctx, cudaGetLastError());
      h3c_status e = exchange(send + off, outs[i] + off, per_peer);
      if (e != H3C_OK) return e;
    }
    H3_CUDA_TRY(ctx, cudaEventRecord(st->in_done[c], x));
    // the previous chunk's output goes back once its attention is done
    if (c > 0) {
      h3c_status e = send_out(c - 1);
      if (e != H3C_OK) return e;
    }
    // the fused call on [P * S_r, hc, D]: every token, this chunk's heads
    H3_CUDA_TRY(ctx, cudaStreamWaitEvent(s, st->in_done[c], 0));
    h3c_attn_args la = a;
    const int64_t ts = (int64_t)hc * 128;
    la.q = h3c_view{qx + off, ts, 128};
    la.k = h3c_view{kx + off, ts, 128};
    la.v = h3c_view{vx + off, ts, 128};
    la.out = h3c_view{ox + off, ts, 128};
    la.heads = hc;
    la.head_offset = 0;
    la.head_count = hc;
    h3c_status e = h3c_attn_fwd(ctx, &la, stream);
    if (e != H3C_OK) return e;
    H3_CUDA_TRY(ctx, cudaEventRecord(st->attn_done[c], s));
  }
  h3c_status e = send_out(nchunk - 1);
  if (e != H3C_OK) return e;
  // rows past seq_len are not computed; they come back as unspecified padding
  H3_CUDA_TRY(ctx, cudaEventRecord(st->out_done, x));
  H3_CUDA_TRY(ctx, cudaStreamWaitEvent(s, st->out_done, 0));
  return H3C_OK;
}

h3c_status h3c_comm_wait(h3c_ctx* ctx, void* stream, int64_t timeout_ms) {
  if (!ctx || timeout_ms < 0) return H3C_ERR_INVALID_ARGUMENT;
  h3c_comm_state* st = comm_of(ctx);
  if (!st) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_comm_wait: no communicator");
  if (st->aborted) return fail(ctx, H3C_ERR_NCCL, "h3c_comm_wait: the communicator was aborted");
  Nccl* n = nccl();
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = (cudaStream_t)stream;
  const double t0 = now_ms();
  auto abort_comm = [&]() {
    if (n && n->CommAbort) n->CommAbort(st->comm);  // stops the communicator's kernels
    st->aborted = true;
  };
  while (true) {
    const cudaError_t q = cudaStreamQuery(s);
    ncclResult_t_ a = kNcclSuccess;
    if (st->nonblocking && n->CommGetAsyncError) n->CommGetAsyncError(st->comm, &a);
    if (a != kNcclSuccess && a != kNcclInProgress) {
      abort_comm();
      return fail(ctx, H3C_ERR_NCCL, std::string("h3c_comm_wait: NCCL reported ") + n->GetErrorString(a));
    }
    if (q == cudaSuccess) return H3C_OK;
    if (q != cudaErrorNotReady) H3_CUDA_TRY(ctx, q);
    if (now_ms() - t0 > (double)timeout_ms) break;
    nap();
  }
  if (!st->nonblocking || !n->CommAbort)
    return fail(ctx, H3C_ERR_TIMEOUT, "h3c_comm_wait: timed out (blocking communicator: cannot abort)");
  abort_comm();
  // the aborted exchange kernels return; let the stream drain (bounded)
  const double t1 = now_ms();
  while (cudaStreamQuery(s) == cudaErrorNotReady && now_ms() - t1 < (double)timeout_ms + 10000.0) nap();
  return fail(ctx, H3C_ERR_TIMEOUT,
              "h3c_comm_wait: a peer did not take part in time; the communicator was aborted (output invalid; "
              "h3c_comm_destroy and h3c_comm_init to continue)");
}

}  // extern "C"
