// The C ABI (include/h3cuda.h): argument checking, the context, the host
// block-mask builder and dispatch to the kernels.  Every entry point returns
// a status; nothing here aborts or exits.
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"

namespace h3 {
cudaError_t launch_rope_table(const int32_t* pos, int32_t seq_len, int3 dims, const float* d_inv, int32_t half,
                              uint16_t* table, cudaStream_t s);
cudaError_t launch_rope_table_shared(const float* pos, int32_t seq_len, const float* d_inv, int32_t n,
                                     uint16_t* table, cudaStream_t s);
cudaError_t launch_mask_build(const h3c_mask_spec& sp, int32_t* counts, int32_t* row_ptr, int32_t* col_idx,
                              int64_t capacity, int64_t* d_nnz, cudaStream_t s);
cudaError_t launch_fill_normal(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream, double mean, double std,
                               int sm_count, cudaStream_t s);
cudaError_t launch_validate_blocks(const int32_t* row_ptr, const int32_t* col_idx, int32_t n_blocks, int64_t nnz,
                                   int32_t* flags, cudaStream_t s);
}  // namespace h3

namespace {

const char* kNullCtxError = "h3c: null context";

h3c_status fail(h3c_ctx* ctx, h3c_status st, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return st;
}

// ------------------------------------------------------------ block mask (host)
int mask_check(const h3c_mask_spec* m) {
  if (!m) return 1;
  if (m->seq_len <= 0 || m->block <= 0 || m->prefix_len < 0 || m->prefix_len > m->seq_len) return 1;
  if ((int64_t)m->frames * m->height * m->width != (int64_t)m->seq_len - m->prefix_len) return 2;
  if (m->frames < 0 || m->height < 0 || m->width < 0) return 2;
  if (m->cell_t <= 0 || m->cell_h <= 0 || m->cell_w <= 0) return 3;
  if (m->radius_t < 0 || m->radius_h < 0 || m->radius_w < 0 || m->n_random < 0) return 4;
  return 0;
}

struct Cell {
  int t, h, w;
};

Cell block_cell(const h3c_mask_spec& m, int b) {
  int64_t v = (int64_t)b * m.block - m.prefix_len;
  int64_t per = (int64_t)m.height * m.width;
  int t = (int)(v / per), rem = (int)(v % per);
  return {t / m.cell_t, (rem / m.width) / m.cell_h, (rem % m.width) / m.cell_w};
}

// Kept key blocks of query block i, ascending.
void mask_row(const h3c_mask_spec& m, int nb, int npb, const std::vector<Cell>& cells, int i,
              std::vector<uint8_t>& row) {
  if (i < npb) {
    std::fill(row.begin(), row.end(), 1);
    return;
  }
  std::fill(row.begin(), row.end(), 0);
  for (int j = 0; j < npb && j < nb; ++j) row[j] = 1;
  const Cell q = cells[i];
  for (int j = npb; j < nb; ++j) {
    const Cell k = cells[j];
    if (std::abs(k.t - q.t) <= m.radius_t && std::abs(k.h - q.h) <= m.radius_h && std::abs(k.w - q.w) <= m.radius_w)
      row[j] = 1;
  }
  uint64_t state = m.seed ^ ((uint64_t)i * 0x9E3779B97F4A7C15ull);
  int added = 0, draws = 64 + 16 * m.n_random;
  for (int a = 0; a < draws && added < m.n_random; ++a) {
    state = h3::splitmix64(state);
    int j = (int)(((state >> 32) * (uint64_t)nb) >> 32);
    if (!row[j]) {
      row[j] = 1;
      ++added;
    }
  }
}

bool view_ok(const h3c_view& v) { return v.ptr && v.token_stride > 0 && v.head_stride > 0; }

// Bytes of workspace the fused path needs: normalised K and Q, [S_pad, Hc, 128] each.
size_t workspace_bytes(const h3c_attn_args& a) {
  if (!(a.flags & H3C_FUSE_PROLOGUE)) return 0;
  size_t s_pad = (size_t)((a.seq_len + 127) / 128) * 128;
  return 2 * s_pad * (size_t)a.head_count * 128 * sizeof(uint16_t);
}

h3c_status check_attn(h3c_ctx* ctx, const h3c_attn_args* a) {
  std::string msg;
  h3c_status st = h3::check_attn_args(a, "h3c_attn_fwd", &msg);
  return st == H3C_OK ? st : fail(ctx, st, msg);
}

}  // namespace

namespace h3 {

h3c_status check_attn_args(const h3c_attn_args* a, const char* who, std::string* msg) {
  auto bad = [&](h3c_status st, const char* why) {
    *msg = std::string(who) + ": " + why;
    return st;
  };
  if (!a) return bad(H3C_ERR_INVALID_ARGUMENT, "null args");
  if (a->head_dim != 128) return bad(H3C_ERR_UNSUPPORTED, "head_dim must be 128");
  if (a->block != 128) return bad(H3C_ERR_UNSUPPORTED, "block must be 128");
  if (a->seq_len <= 0 || a->heads <= 0 || a->head_count <= 0 || a->head_offset < 0 ||
      a->head_offset + a->head_count > a->heads)
    return bad(H3C_ERR_INVALID_ARGUMENT, "bad seq_len/heads/head range");
  if (!view_ok(a->q) || !view_ok(a->k) || !view_ok(a->v) || !view_ok(a->out))
    return bad(H3C_ERR_INVALID_ARGUMENT, "null pointer or non-positive stride in q/k/v/out");
  if (!a->row_ptr || !a->col_idx) return bad(H3C_ERR_INVALID_ARGUMENT, "null block list");
  if (!(a->scale > 0.f) || !std::isfinite(a->scale))
    return bad(H3C_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  if (a->flags & H3C_FUSE_PROLOGUE) {
    if (!a->q_norm_weight || !a->k_norm_weight)
      return bad(H3C_ERR_INVALID_ARGUMENT, "fused prologue needs q/k norm weights");
    if (!(a->flags & H3C_NO_ROPE)) {
      if (!a->rope_table) return bad(H3C_ERR_INVALID_ARGUMENT, "fused prologue needs a rope table");
      if (a->rope_half <= 0 || 2 * a->rope_half > 128) return bad(H3C_ERR_UNSUPPORTED, "rope_half must be in [1, 64]");
    }
    if (!(a->eps >= 0.f) || !std::isfinite(a->eps)) return bad(H3C_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
    if (((uintptr_t)a->q_norm_weight & 15) || ((uintptr_t)a->k_norm_weight & 15) || ((uintptr_t)a->rope_table & 7))
      return bad(H3C_ERR_UNSUPPORTED, "norm weights need 16-byte, the rope table 8-byte alignment");
  }
  // 16-byte aligned rows are required by the vectorised and TMA loads.
  const h3c_view* vs[4] = {&a->q, &a->k, &a->v, &a->out};
  for (const h3c_view* v : vs) {
    if (((uintptr_t)v->ptr & 15) || (v->token_stride & 7) || (v->head_stride & 7))
      return bad(H3C_ERR_UNSUPPORTED, "operands need 16-byte aligned rows");
  }
  return H3C_OK;
}

}  // namespace h3

extern "C" {

int h3c_abi_version(void) { return H3C_ABI_VERSION; }

h3c_status h3c_device_count(int* count) {
  if (!count) return H3C_ERR_INVALID_ARGUMENT;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
  *count = n;
  return H3C_OK;
}

h3c_status h3c_init(int device, h3c_ctx** out) {
  if (!out) return H3C_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return H3C_ERR_NO_DEVICE;
  h3c_ctx* ctx = new (std::nothrow) h3c_ctx();
  if (!ctx) return H3C_ERR_CAPACITY;
  ctx->device = device;
  if (cudaSetDevice(device) != cudaSuccess || cudaGetDeviceProperties(&ctx->prop, device) != cudaSuccess) {
    delete ctx;
    return H3C_ERR_CUDA;
  }
  if (ctx->prop.major != 10) {  // sm_100 family only; the kernels are built for sm_100a
    delete ctx;
    return H3C_ERR_NO_DEVICE;
  }
  if (cudaMalloc(&ctx->d_counter, 64) != cudaSuccess || cudaMemset(ctx->d_counter, 0, 64) != cudaSuccess ||
      cudaEventCreateWithFlags(&ctx->workspace_done, cudaEventDisableTiming) != cudaSuccess) {
    if (ctx->d_counter) cudaFree(ctx->d_counter);
    delete ctx;
    return H3C_ERR_CUDA;
  }
  *out = ctx;
  return H3C_OK;
}

h3c_status h3c_destroy(h3c_ctx* ctx) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  h3c_comm_destroy(ctx);
  cudaSetDevice(ctx->device);
  if (ctx->workspace_done) cudaEventSynchronize(ctx->workspace_done);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->workspace_done) cudaEventDestroy(ctx->workspace_done);
  if (ctx->d_counter) cudaFree(ctx->d_counter);
  delete ctx;
  return H3C_OK;
}

h3c_status h3c_device_alloc(h3c_ctx* ctx, size_t bytes, void** out) {
  if (!ctx || !out) return H3C_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  if (bytes == 0) return H3C_OK;
  cudaError_t e = cudaMalloc(out, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(ctx, H3C_ERR_CAPACITY, "h3c_device_alloc: out of device memory");
  }
  H3_CUDA_TRY(ctx, e);
  return H3C_OK;
}

h3c_status h3c_device_free(h3c_ctx* ctx, void* ptr) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!ptr) return H3C_OK;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  H3_CUDA_TRY(ctx, cudaFree(ptr));
  return H3C_OK;
}

const char* h3c_last_error(const h3c_ctx* ctx) { return ctx ? ctx->err.c_str() : kNullCtxError; }

h3c_status h3c_device_info(h3c_ctx* ctx, h3c_devinfo* info) {
  if (!ctx || !info) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_device_info: null argument");
  std::memset(info, 0, sizeof(*info));
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  info->device = ctx->device;
  info->cc_major = ctx->prop.major;
  info->cc_minor = ctx->prop.minor;
  info->sm_count = ctx->prop.multiProcessorCount;
  info->hbm_bytes = (int64_t)ctx->prop.totalGlobalMem;
  size_t fr = 0, tot = 0;
  H3_CUDA_TRY(ctx, cudaMemGetInfo(&fr, &tot));
  info->hbm_free_bytes = (int64_t)fr;
  info->max_smem_per_block_optin = (int32_t)ctx->prop.sharedMemPerBlockOptin;
  info->l2_bytes = ctx->prop.l2CacheSize;
  int n = 0;
  H3_CUDA_TRY(ctx, cudaGetDeviceCount(&n));
  for (int d = 0; d < n && d < 31; ++d) {
    if (d == ctx->device) continue;
    int ok = 0;
    if (cudaDeviceCanAccessPeer(&ok, ctx->device, d) == cudaSuccess && ok) {
      info->peer_count++;
      info->nvlink_peer_mask |= (1 << d);
    }
  }
  std::memcpy(info->name, ctx->prop.name, sizeof(info->name) - 1);
  for (int d = 0; d < n && d < 31; ++d) {
    int atomics = 0;
    if (d != ctx->device &&
        cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, ctx->device, d) == cudaSuccess &&
        atomics)
      info->native_atomic_peer_mask |= (1 << d);
  }
  H3_CUDA_TRY(ctx, cudaDeviceGetPCIBusId(info->pci_bus_id, (int)sizeof(info->pci_bus_id), ctx->device));
  h3c_nvlink nv;
  info->nvlink_links = info->nvlink_version = info->nvswitch_links = -1;
  if (h3c_nvlink_query(info->pci_bus_id, &nv) == H3C_OK) {
    info->nvlink_links = nv.links_active;
    info->nvlink_version = nv.version;
    info->nvswitch_links = nv.links_to_switch;
  }
  return H3C_OK;
}

h3c_status h3c_blockmask_build(const h3c_mask_spec* spec, int32_t* row_ptr, int32_t* col_idx, int64_t capacity,
                               int64_t* nnz) {
  int st = mask_check(spec);
  if (st == 2) return H3C_ERR_UNSUPPORTED;
  if (st) return H3C_ERR_INVALID_ARGUMENT;
  if (col_idx && capacity < 0) return H3C_ERR_INVALID_ARGUMENT;
  const h3c_mask_spec& m = *spec;
  const int nb = (m.seq_len + m.block - 1) / m.block;
  const int npb = (m.prefix_len + m.block - 1) / m.block;
  std::vector<Cell> cells(nb);
  for (int b = npb; b < nb; ++b) cells[b] = block_cell(m, b);
  std::vector<uint8_t> row(nb);
  int64_t off = 0;
  if (row_ptr) row_ptr[0] = 0;
  bool overflow = false;
  for (int i = 0; i < nb; ++i) {
    mask_row(m, nb, npb, cells, i, row);
    for (int j = 0; j < nb; ++j)
      if (row[j]) {
        if (col_idx) {
          if (off < capacity) col_idx[off] = j;
          else overflow = true;
        }
        ++off;
      }
    if (row_ptr) row_ptr[i + 1] = (int32_t)off;
  }
  if (nnz) *nnz = off;
  return overflow ? H3C_ERR_CAPACITY : H3C_OK;
}

h3c_status h3c_blockmask_build_device(h3c_ctx* ctx, const h3c_mask_spec* spec, int32_t* d_row_ptr,
                                      int32_t* d_col_idx, int64_t capacity, int64_t* nnz, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  int st = mask_check(spec);
  if (st == 2) return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_blockmask_build_device: lattice does not fill the video span");
  if (st) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_blockmask_build_device: invalid spec");
  if (!d_row_ptr || !d_col_idx || capacity <= 0)
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_blockmask_build_device: null output or capacity");
  const int nb = (spec->seq_len + spec->block - 1) / spec->block;
  if (nb > 48 * 1024 * 8) return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_blockmask_build_device: too many blocks");
  cudaStream_t s = (cudaStream_t)stream;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int32_t* counts = nullptr;
  H3_CUDA_TRY(ctx, cudaMallocAsync((void**)&counts, sizeof(int32_t) * (nb + 1), s));
  cudaError_t e = h3::launch_mask_build(*spec, counts, d_row_ptr, d_col_idx, capacity, ctx->d_counter, s);
  cudaFreeAsync(counts, s);
  H3_CUDA_TRY(ctx, e);
  int64_t total = 0;
  H3_CUDA_TRY(ctx, cudaMemcpyAsync(&total, ctx->d_counter, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  H3_CUDA_TRY(ctx, cudaStreamSynchronize(s));
  if (nnz) *nnz = total;
  if (total > capacity) return fail(ctx, H3C_ERR_CAPACITY, "h3c_blockmask_build_device: col_idx capacity too small");
  return H3C_OK;
}

h3c_status h3c_rope_table(h3c_ctx* ctx, const int32_t* d_pos, int32_t seq_len, const int32_t dims[3], double theta,
                          void* d_table, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!d_pos || !dims || !d_table || seq_len < 0 || !(theta > 0))
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_rope_table: invalid argument");
  for (int a = 0; a < 3; ++a)
    if (dims[a] < 0 || (dims[a] & 1)) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_rope_table: dims must be even");
  const int half = (dims[0] + dims[1] + dims[2]) / 2;
  if (half <= 0 || half > 64) return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_rope_table: 2*half must be in [2, 128]");
  float inv[64];
  int n = 0;
  for (int a = 0; a < 3; ++a)
    for (int k = 0; k < dims[a] / 2; ++k) inv[n++] = (float)std::pow(theta, -2.0 * (double)k / (double)dims[a]);
  cudaStream_t s = (cudaStream_t)stream;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  float* d_inv = nullptr;
  H3_CUDA_TRY(ctx, cudaMallocAsync((void**)&d_inv, sizeof(inv), s));
  cudaError_t e = cudaMemcpyAsync(d_inv, inv, sizeof(float) * half, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = h3::launch_rope_table(d_pos, seq_len, make_int3(dims[0], dims[1], dims[2]), d_inv, half, (uint16_t*)d_table, s);
  cudaError_t e2 = cudaStreamSynchronize(s);  // the host copy source lives on this stack frame
  cudaFreeAsync(d_inv, s);
  H3_CUDA_TRY(ctx, e);
  H3_CUDA_TRY(ctx, e2);
  return H3C_OK;
}

h3c_status h3c_rope_table_shared(h3c_ctx* ctx, const float* d_pos, int32_t seq_len, const float* d_inv_freq,
                                 int32_t n, void* d_table, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!d_pos || !d_inv_freq || !d_table || seq_len < 0 || n <= 0)
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_rope_table_shared: invalid argument");
  if (3 * n > 64) return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_rope_table_shared: 3*n must be <= 64");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  H3_CUDA_TRY(ctx, h3::launch_rope_table_shared(d_pos, seq_len, d_inv_freq, n, (uint16_t*)d_table,
                                                (cudaStream_t)stream));
  return H3C_OK;
}

h3c_status h3c_prologue(h3c_ctx* ctx, h3c_view x, h3c_view out, int32_t seq_len, int32_t heads, int32_t head_offset,
                        int32_t head_count, const void* norm_weight, float eps, const void* rope_table,
                        int32_t rope_half, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!view_ok(x) || !view_ok(out) || !norm_weight || seq_len < 0 || heads <= 0 || head_offset < 0 ||
      head_count <= 0 || head_offset + head_count > heads || !(eps >= 0.f))
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_prologue: invalid argument");
  if (rope_table && (rope_half <= 0 || 2 * rope_half > 128))
    return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_prologue: rope_half must be in [1, 64]");
  if (((uintptr_t)x.ptr & 15) || ((uintptr_t)out.ptr & 15) || (x.token_stride & 7) || (x.head_stride & 7) ||
      (out.token_stride & 7) || (out.head_stride & 7) || ((uintptr_t)norm_weight & 15) ||
      ((uintptr_t)rope_table & 7))
    return fail(ctx, H3C_ERR_UNSUPPORTED, "h3c_prologue: rows, weight and table need 16/16/8-byte alignment");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  const uint16_t* xp = (const uint16_t*)x.ptr + (int64_t)head_offset * x.head_stride;
  uint16_t* yp = (uint16_t*)out.ptr + (int64_t)head_offset * out.head_stride;
  H3_CUDA_TRY(ctx, h3::launch_prologue(xp, x.token_stride, x.head_stride, yp, out.token_stride, out.head_stride,
                                       seq_len, head_count, (const uint16_t*)norm_weight, eps,
                                       (const uint16_t*)rope_table, rope_table ? rope_half : 0,
                                       (cudaStream_t)stream));
  return H3C_OK;
}

h3c_status h3c_attn_workspace_size(const h3c_attn_args* args, size_t* bytes) {
  if (!args || !bytes) return H3C_ERR_INVALID_ARGUMENT;
  *bytes = workspace_bytes(*args);
  return H3C_OK;
}

h3c_status h3c_attn_fwd(h3c_ctx* ctx, const h3c_attn_args* args, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  h3c_status st = check_attn(ctx, args);
  if (st != H3C_OK) return st;
  const h3c_attn_args& a = *args;
  cudaStream_t s = (cudaStream_t)stream;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));

  h3::AttnLaunch L{};
  const int64_t ho = a.head_offset;
  L.q = (const uint16_t*)a.q.ptr + ho * a.q.head_stride; L.q_tok = a.q.token_stride; L.q_head = a.q.head_stride;
  L.k = (const uint16_t*)a.k.ptr + ho * a.k.head_stride; L.k_tok = a.k.token_stride; L.k_head = a.k.head_stride;
  L.v = (const uint16_t*)a.v.ptr + ho * a.v.head_stride; L.v_tok = a.v.token_stride; L.v_head = a.v.head_stride;
  L.o = (uint16_t*)a.out.ptr + ho * a.out.head_stride; L.o_tok = a.out.token_stride; L.o_head = a.out.head_stride;
  L.seq_len = a.seq_len;
  L.n_blocks = (a.seq_len + 127) / 128;
  L.head_count = a.head_count;
  L.scale_log2 = a.scale * 1.4426950408889634f;
  L.row_ptr = a.row_ptr;
  L.col_idx = a.col_idx;

  if (a.flags & H3C_FUSE_PROLOGUE) {
    size_t need = workspace_bytes(a);
    if (ctx->workspace_bytes < need) {
      if (ctx->workspace) {
        // the last launch that read the old workspace may run on another
        // stream: wait for it, then release the buffer
        H3_CUDA_TRY(ctx, cudaEventSynchronize(ctx->workspace_done));
        cudaFree(ctx->workspace);
        ctx->workspace = nullptr;
        ctx->workspace_bytes = 0;
      }
      H3_CUDA_TRY(ctx, cudaMalloc(&ctx->workspace, need));
      ctx->workspace_bytes = need;
    }
    // normalised K (and Q) in [S_pad, Hc, 128] layout inside the workspace
    const size_t s_pad = (size_t)L.n_blocks * 128;
    uint16_t* kn = (uint16_t*)ctx->workspace;
    uint16_t* qn = kn + s_pad * (size_t)a.head_count * 128;
    const uint16_t* table = (a.flags & H3C_NO_ROPE) ? nullptr : (const uint16_t*)a.rope_table;
    const int half = table ? a.rope_half : 0;
    H3_CUDA_TRY(ctx, h3::launch_prologue_qk(L.q, L.q_tok, L.q_head, qn, L.k, L.k_tok, L.k_head, kn,
                                            (int64_t)a.head_count * 128, a.seq_len, a.head_count,
                                            (const uint16_t*)a.q_norm_weight, (const uint16_t*)a.k_norm_weight,
                                            a.eps, table, half, ctx->prop.multiProcessorCount, s));
    L.k = kn; L.k_tok = (int64_t)a.head_count * 128; L.k_head = 128;
    L.q = qn; L.q_tok = (int64_t)a.head_count * 128; L.q_head = 128;
  }

  L.status = (int32_t*)(ctx->d_counter + 1);
  L.wait_limit_ns = 4000000000ull;
  L.drop_item = -1;
  L.pdl = (a.flags & H3C_FUSE_PROLOGUE) ? 1 : 0;
  // Test hooks (fault injection on the host side): a K/V load the producer
  // skips, so that the consumers' bounded waits run out, and a shorter bound.
  if (const char* d = getenv("H3C_TEST_DROP_ITEM")) L.drop_item = atoi(d);
  if (const char* w = getenv("H3C_TEST_WAIT_LIMIT_NS")) L.wait_limit_ns = strtoull(w, nullptr, 10);
  cudaError_t e;
  if (a.flags & H3C_KERNEL_MMA_SYNC) {
    e = h3::launch_attn_mma(L, s);
  } else {
    std::string why;
    e = h3::launch_attn_tc(L, s, &why);
    if (e != cudaSuccess) return fail(ctx, H3C_ERR_CUDA, "tcgen05 attention: " + why + cudaGetErrorString(e));
  }
  H3_CUDA_TRY(ctx, e);
  if (a.flags & H3C_FUSE_PROLOGUE) H3_CUDA_TRY(ctx, cudaEventRecord(ctx->workspace_done, s));
  return H3C_OK;
}

h3c_status h3c_blockmask_validate(h3c_ctx* ctx, const int32_t* d_row_ptr, const int32_t* d_col_idx,
                                  int32_t n_blocks, int64_t nnz, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!d_row_ptr || (!d_col_idx && nnz > 0) || n_blocks <= 0 || nnz < 0 || nnz > INT32_MAX)
    return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_blockmask_validate: invalid argument");
  cudaStream_t s = (cudaStream_t)stream;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int32_t* flags = (int32_t*)(ctx->d_counter + 2);
  H3_CUDA_TRY(ctx, h3::launch_validate_blocks(d_row_ptr, d_col_idx, n_blocks, nnz, flags, s));
  int32_t bad = 0;
  H3_CUDA_TRY(ctx, cudaMemcpyAsync(&bad, flags, sizeof(bad), cudaMemcpyDeviceToHost, s));
  H3_CUDA_TRY(ctx, cudaStreamSynchronize(s));
  if (!bad) return H3C_OK;
  std::string why = "h3c_blockmask_validate:";
  if (bad & 1) why += " row_ptr[0] != 0 or row_ptr[n_blocks] != nnz;";
  if (bad & 2) why += " row_ptr decreasing or outside [0, nnz];";
  if (bad & 4) why += " a column index outside [0, n_blocks);";
  if (bad & 8) why += " columns of a row not strictly ascending;";
  return fail(ctx, H3C_ERR_INVALID_ARGUMENT, why);
}

h3c_status h3c_attn_fwd_sync(h3c_ctx* ctx, const h3c_attn_args* args, void* stream) {
  h3c_status st = h3c_attn_fwd(ctx, args, stream);
  if (st != H3C_OK) return st;
  H3_CUDA_TRY(ctx, cudaStreamSynchronize((cudaStream_t)stream));
  return h3c_device_status(ctx);
}

h3c_status h3c_device_status(h3c_ctx* ctx) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int32_t word = 0;
  H3_CUDA_TRY(ctx, cudaMemcpy(&word, ctx->d_counter + 1, sizeof(word), cudaMemcpyDeviceToHost));
  if (word == 0) return H3C_OK;
  H3_CUDA_TRY(ctx, cudaMemset(ctx->d_counter + 1, 0, sizeof(int64_t)));
  return fail(ctx, (h3c_status)word, "h3c_attn_fwd: a bounded device wait gave up (H3C_ERR_TIMEOUT); output invalid");
}

h3c_status h3c_fill_normal_bf16(h3c_ctx* ctx, void* d_out, int64_t n, uint64_t seed, uint64_t stream_id, double mean,
                                double std, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!d_out || n < 0) return fail(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_fill_normal_bf16: invalid argument");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  H3_CUDA_TRY(ctx, h3::launch_fill_normal((uint16_t*)d_out, n, seed, stream_id, mean, std,
                                          ctx->prop.multiProcessorCount, (cudaStream_t)stream));
  return H3C_OK;
}

}  // extern "C"
