/*
 * h3cuda.h -- C ABI of the B200 (sm_100a) H3 self-attention hot path.
 *
 * This is the boundary a Swift `CUDABackend: H3AttentionBackend` (module
 * CH3Cuda) or any ctypes / cffi caller binds.  Plain pointers and sizes only;
 * no C++ or torch types.  Every call returns an h3c_status and never aborts;
 * h3c_last_error() gives the message of the last failure on a context.
 *
 * What each entry point replaces in the reference (MiniMax-H3-Swift):
 *   h3c_attn_fwd          H3AttentionBackend.attend + AttentionLayer.sdpa
 *                         (Sources/H3Attention/AttentionBackend.swift:126-127,
 *                          Sources/H3Modules/DiTBlock.swift:293-328); with
 *                         H3C_FUSE_PROLOGUE it also covers the per-head
 *                         qNorm/kNorm and SplitHalfRoPE of
 *                         AttentionLayer.callAsFunction (DiTBlock.swift:346-352)
 *   h3c_prologue          H3RMSNorm (Sources/H3Modules/Modulation.swift:116-120)
 *                         + SplitHalfRoPE.apply (DiTBlock.swift:83-103);
 *                         the unfused bisection kernel
 *   h3c_rope_table        H3RoPE.angles + rotationTable
 *                         (Sources/H3Modules/H3Transformer.swift:62-78),
 *                         built once per render in prepareRender (:263-276)
 *   h3c_rope_table_shared the same table as the production transformer builds
 *                         it: float PackedLayout.positionIds and the
 *                         checkpoint's shared rope.inv_freq (H3Transformer.
 *                         swift:62-78, :270-273; PackedSequence.swift:186)
 *   h3c_packed_layout     PackedLayout.init segment table (Sources/H3Foundation/
 *                         PackedSequence.swift:192-297), host only
 *   h3c_packed_positions_device  PackedLayout.positionIds narrowed to fp32
 *                         (H3Transformer.swift:270), evaluated on the device
 *   h3c_rope_table_layout positions + H3RoPE table in one kernel: what
 *                         prepareRender builds (H3Transformer.swift:263-276)
 *   h3c_blockmask_build   new: the compacted 128x128 block list (no reference
 *                         counterpart; prefix rule of AxialTopology.allows,
 *                         Sources/H3Attention/AxialTopology.swift:128-137)
 *   h3c_blockmask_validate the refusal of a malformed mask, as
 *                         AxialTopology.validate refuses mismatched geometry
 *                         (Sources/H3Attention/AxialTopology.swift:67-70)
 *   h3c_device_info       H3Hardware Machine.detect (Sources/H3Hardware/
 *                         Machine.swift:48-56), for CUDA devices and NVLink
 *   h3c_nvlink_query      the NVLink / NVSwitch part of that discovery
 *                         (Machine.swift:48-56 measures, never assumes)
 *   h3c_init/h3c_destroy  the backend instance AttentionRegistry.resolve
 *                         creates once per render (AttentionBackend.swift:255-259)
 */
#ifndef H3CUDA_H
#define H3CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3C_ABI_VERSION 2

typedef enum h3c_status {
  H3C_OK = 0,
  H3C_ERR_INVALID_ARGUMENT = 1,   /* null pointer, negative size, bad stride */
  H3C_ERR_UNSUPPORTED = 2,        /* geometry the kernels decline (e.g. head_dim != 128) */
  H3C_ERR_CUDA = 3,               /* a CUDA runtime / driver call failed */
  H3C_ERR_NCCL = 4,               /* reserved for the sequence-sharded path */
  H3C_ERR_TIMEOUT = 5,            /* a bounded device wait gave up */
  H3C_ERR_CAPACITY = 6,           /* caller buffer or fixed limit too small */
  H3C_ERR_NO_DEVICE = 7           /* no sm_100 device, or the device is not usable */
} h3c_status;

typedef struct h3c_ctx h3c_ctx;

/* Device discovery (the CUDA counterpart of H3Hardware.Machine). */
typedef struct h3c_devinfo {
  int32_t device;
  int32_t cc_major, cc_minor;
  int32_t sm_count;
  int64_t hbm_bytes;
  int64_t hbm_free_bytes;
  int32_t max_smem_per_block_optin;
  int32_t l2_bytes;
  int32_t peer_count;         /* devices this one can access peer-to-peer (NVLink or PCIe) */
  int32_t nvlink_peer_mask;   /* bit d set: device d is a P2P peer (cudaDeviceCanAccessPeer) */
  char name[96];
  /* from NVML (read-only queries); -1 where NVML is not available */
  int32_t nvlink_links;       /* active NVLink links of this device */
  int32_t nvlink_version;     /* NVLink version NVML reports for the first active link */
  int32_t nvswitch_links;     /* active links whose remote end is an NVSwitch */
  int32_t native_atomic_peer_mask; /* bit d: P2P native atomics with device d (NVLink, not PCIe) */
  char pci_bus_id[16];        /* "0000:1B:00.0" */
} h3c_devinfo;

/* NVLink state of one device, by PCI bus id (NVML through dlopen; nothing is
 * changed).  available = 0 when NVML cannot be loaded. */
typedef struct h3c_nvlink {
  int32_t available;
  int32_t links_active;
  int32_t links_to_switch;
  int32_t links_to_gpu;
  int32_t version;            /* -1: unknown */
} h3c_nvlink;

/* Block-mask specification (128x128 blocks in raster token order).
 * Tokens [0, prefix_len) are the conditioning prefix (e.g. audio); tokens
 * [prefix_len, seq_len) are a frames x height x width video lattice in t-major,
 * h, w order.  Query block i (blocks touching the prefix keep every key
 * block) keeps: every prefix key block; every video key block whose coarse
 * cell (t/cell_t, h/cell_h, w/cell_w of the block's first token) lies within
 * (radius_t, radius_h, radius_w) of its own; then n_random distinct extra key
 * blocks drawn with splitmix64 from seed ^ (i * 0x9E3779B97F4A7C15). */
typedef struct h3c_mask_spec {
  int32_t seq_len, block, prefix_len;
  int32_t frames, height, width;
  int32_t cell_t, cell_h, cell_w;
  int32_t radius_t, radius_h, radius_w;
  int32_t n_random;
  uint64_t seed;
} h3c_mask_spec;

/* A bf16 [tokens, heads, 128] operand: element (s, h, d) sits at
 * ptr[s * token_stride + h * head_stride + d].  [S,H,D] has
 * (token_stride, head_stride) = (H*D, D); the seam's [H,S,D] has (D, S*D). */
typedef struct h3c_view {
  void* ptr;
  int64_t token_stride;
  int64_t head_stride;
} h3c_view;

enum {
  H3C_FUSE_PROLOGUE = 1,      /* q, k are pre-norm; apply RMSNorm + RoPE */
  H3C_KERNEL_MMA_SYNC = 2,    /* force the mma.sync bisection kernel */
  H3C_NO_ROPE = 4             /* with H3C_FUSE_PROLOGUE: RMSNorm only */
};

typedef struct h3c_attn_args {
  h3c_view q, k, v, out;      /* bf16 device memory; out may not alias q/k/v */
  int32_t seq_len;            /* S (valid tokens) */
  int32_t heads;              /* heads present in the views */
  int32_t head_dim;           /* must be 128 */
  int32_t head_offset;        /* process heads [head_offset, head_offset+head_count) */
  int32_t head_count;
  float scale;                /* softmax scale, 1/sqrt(head_dim) in H3 */
  const int32_t* row_ptr;     /* device CSR of the block mask: [n_blocks+1] */
  const int32_t* col_idx;     /* device, ascending within each row */
  int32_t block;              /* must be 128 */
  int32_t flags;              /* H3C_* flags above */
  /* prologue (read when H3C_FUSE_PROLOGUE is set) */
  const void* q_norm_weight;  /* bf16 [128] */
  const void* k_norm_weight;  /* bf16 [128] */
  float eps;
  const void* rope_table;     /* bf16 [S, rope_half, 4]: (c, -s, s, c) */
  int32_t rope_half;          /* rotated pairs; 2*rope_half <= 128 */
} h3c_attn_args;

/* --- lifecycle --------------------------------------------------------- */
int h3c_abi_version(void);
h3c_status h3c_init(int device, h3c_ctx** out);
h3c_status h3c_destroy(h3c_ctx* ctx);
const char* h3c_last_error(const h3c_ctx* ctx);   /* never NULL */
h3c_status h3c_device_info(h3c_ctx* ctx, h3c_devinfo* info);
h3c_status h3c_device_count(int* count);
/* NVLink links of the device at pci_bus_id: H3C_OK, H3C_ERR_NO_DEVICE (NVML
 * does not know the bus id) or H3C_ERR_UNSUPPORTED (no NVML).  Needs no
 * context and no CUDA call. */
h3c_status h3c_nvlink_query(const char* pci_bus_id, h3c_nvlink* out);

/* Device memory on the context's device, for hosts that bind no CUDA runtime
 * of their own (a Swift host keeps its block list and RoPE table here).
 * h3c_device_free(ctx, NULL) is a no-op.  The reference has no counterpart:
 * MLX owns its buffers (Sources/H3Attention/AttentionBackend.swift:126-127
 * takes MLXArrays). */
h3c_status h3c_device_alloc(h3c_ctx* ctx, size_t bytes, void** out);
h3c_status h3c_device_free(h3c_ctx* ctx, void* ptr);

/* --- block mask ---------------------------------------------------------- */
/* Host builder.  row_ptr: [n_blocks+1] or NULL; col_idx: capacity entries or
 * NULL (query nnz first).  n_blocks = ceil(seq_len / block). */
h3c_status h3c_blockmask_build(const h3c_mask_spec* spec, int32_t* row_ptr, int32_t* col_idx,
                               int64_t capacity, int64_t* nnz);
/* Checks a caller's device block list before it is used: row_ptr[0] == 0,
 * row_ptr non-decreasing with row_ptr[n_blocks] == nnz (no col_idx entry past
 * nnz is read), every column in [0, n_blocks) and strictly ascending within
 * its row.  The attention kernels trust the list (an unsorted or out-of-range
 * list gives wrong output, not a fault, as TMA fills out-of-range tiles with
 * zeros), so a caller that builds its own lists validates them once here.
 * H3C_ERR_INVALID_ARGUMENT with the reasons in h3c_last_error otherwise.
 * Synchronises `stream`. */
h3c_status h3c_blockmask_validate(h3c_ctx* ctx, const int32_t* d_row_ptr, const int32_t* d_col_idx, int32_t n_blocks,
                                  int64_t nnz, void* stream);
/* Device builder, bit-identical to the host one.  d_row_ptr [n_blocks+1] and
 * d_col_idx [capacity] are device memory; *nnz is written on the host after a
 * stream synchronise.  Asynchronous otherwise. */
h3c_status h3c_blockmask_build_device(h3c_ctx* ctx, const h3c_mask_spec* spec, int32_t* d_row_ptr,
                                      int32_t* d_col_idx, int64_t capacity, int64_t* nnz,
                                      void* stream);

/* --- prologue and rope ---------------------------------------------------- */
/* RoPE table on the device from integer positions d_pos [S,3] (t,h,w):
 * dims = rotary channels per axis (sum = 2*half), theta as H3RoPE. */
h3c_status h3c_rope_table(h3c_ctx* ctx, const int32_t* d_pos, int32_t seq_len, const int32_t dims[3],
                          double theta, void* d_table, void* stream);
/* RoPE table from float positions d_pos [S,3] (t,h,w; fractional values
 * allowed, as PackedLayout makes them) and ONE shared inverse-frequency
 * vector d_inv_freq [n] (the checkpoint's rope.inv_freq) applied to each
 * axis: half = 3n pairs, angle(s, a*n+k) = pos[s,a] * inv[k] in fp32,
 * entry (c, -s, s, c) rounded to bf16.  All pointers are device memory;
 * no allocation, no synchronisation (stream-ordered).  3n <= 64. */
h3c_status h3c_rope_table_shared(h3c_ctx* ctx, const float* d_pos, int32_t seq_len, const float* d_inv_freq,
                                 int32_t n, void* d_table, void* stream);
/* --- packed layout (PackedSequence.swift) -------------------------------- */
/* Segment kinds, in SegmentKind's order (PackedSequence.swift:20-27). */
enum { H3C_SEG_TEXT = 0, H3C_SEG_COND = 1, H3C_SEG_REF_IMAGE = 2, H3C_SEG_REF_AUDIO = 3, H3C_SEG_AUDIO = 4,
       H3C_SEG_VIDEO = 5 };
/* ReferenceKind (PackedSequence.swift:157-162). */
enum { H3C_REF_IMAGE = 0, H3C_REF_AUDIO = 1, H3C_REF_VIDEO = 2, H3C_REF_VIDEO_AUDIO = 3 };

typedef struct {          /* ReferenceBlock */
  int32_t kind, latent_h, latent_w, latent_t, ref_audio_t;
} h3c_ref_block;

typedef struct {          /* PackedLayout(textTokens:geometry:keyframes:refs:) */
  int32_t text_tokens;
  int32_t frame_count, latent_t, audio_t, latent_h, latent_w;  /* LatentGeometry */
  int32_t patch;                      /* H3Config.patchSize[1] (2) */
  int32_t n_keyframes;
  const int32_t* keyframes;           /* resolved pixel frame indices */
  int32_t n_refs;
  const h3c_ref_block* refs;
} h3c_layout_spec;

typedef struct { int32_t start, stop, kind; } h3c_segment;

/* Segment table and total rows of the packed sequence (host only).  An
 * anchor off the timeline or an axis smaller than the patch is refused with
 * H3C_ERR_INVALID_ARGUMENT and the reason in err (the reference throws
 * H3Error there; err may be NULL).  capacity 0 queries the counts; a smaller
 * non-zero capacity returns H3C_ERR_CAPACITY. */
h3c_status h3c_packed_layout(const h3c_layout_spec* spec, h3c_segment* segments, int32_t capacity,
                             int32_t* n_segments, int64_t* total_tokens, char* err, size_t err_len);
/* d_pos [S, 3] fp32 = Float(positionIds), bit-identical to the reference's
 * float64 construction narrowed to fp32.  capacity in tokens.  At most 40
 * segments.  Stream-ordered, no allocation. */
h3c_status h3c_packed_positions_device(h3c_ctx* ctx, const h3c_layout_spec* spec, float* d_pos, int64_t capacity,
                                       void* stream);
/* d_table [S, 3n, 4] bf16 from the layout's positions and the shared
 * d_inv_freq [n] (equal to h3c_packed_positions_device followed by
 * h3c_rope_table_shared, without the positions buffer). */
h3c_status h3c_rope_table_layout(h3c_ctx* ctx, const h3c_layout_spec* spec, const float* d_inv_freq, int32_t n,
                                 void* d_table, int64_t capacity, void* stream);

/* out = SplitHalfRoPE(RMSNorm(x)) for one operand (q or k), rows (s, h) for
 * h in [head_offset, head_offset+head_count).  table NULL: RMSNorm only. */
h3c_status h3c_prologue(h3c_ctx* ctx, h3c_view x, h3c_view out, int32_t seq_len, int32_t heads,
                        int32_t head_offset, int32_t head_count, const void* norm_weight, float eps,
                        const void* rope_table, int32_t rope_half, void* stream);

/* --- attention ------------------------------------------------------------ */
/* Block-sparse attention forward, asynchronous on `stream` (a cudaStream_t,
 * NULL = legacy default stream).  With H3C_FUSE_PROLOGUE the context's
 * workspace holds the normalised queries and keys (grown on demand with
 * cudaMalloc; before a larger buffer replaces it the call waits for the last
 * launch that read the old one, on whatever stream that ran).  A context
 * serves one stream at a time: fused calls of one context on two streams
 * without ordering between them race on its workspace and status word; use
 * one context per concurrent stream. */
h3c_status h3c_attn_fwd(h3c_ctx* ctx, const h3c_attn_args* args, void* stream);
/* Bytes of workspace h3c_attn_fwd needs for these args. */
h3c_status h3c_attn_workspace_size(const h3c_attn_args* args, size_t* bytes);
/* Reads (and clears) the status word the attention kernel writes when one of
 * its bounded device waits gives up: H3C_OK, or H3C_ERR_TIMEOUT (the output
 * of that call is invalid; the context stays usable).  Synchronous.  The
 * bounded waits replace the reference's render-level cancellation
 * (Sources/MiniMaxH3/RenderEngine.swift:574-590) at the kernel level. */
h3c_status h3c_device_status(h3c_ctx* ctx);
/* Synchronous helper for tests: h3c_attn_fwd, a stream synchronise, then
 * h3c_device_status. */
h3c_status h3c_attn_fwd_sync(h3c_ctx* ctx, const h3c_attn_args* args, void* stream);
/* Allocation-free variant of the fused path (H3C_FUSE_PROLOGUE required), for
 * callers that may not call cudaMalloc (their process hands device memory to
 * its own pool, or an allocation at call time is unacceptable).  No context:
 * runs on the current device.  Its scratch (normalised Q and K) is a fixed
 * 32 MiB device array inside the library, held by every GPU that loads it;
 * ceil(S/128)*128 * head_count must be <= 65536, else H3C_ERR_CAPACITY.  The
 * first call on a device resolves the array's address (make it before any
 * stream capture).  All calls share the array: calls that overlap on the GPU
 * race.  err (optional, err_len bytes) receives the message of a failure.
 * A bounded device wait that gives up is recorded in a second fixed device
 * word of the library, cleared at the start of every call: read it with
 * h3c_attn_fwd_noalloc_status.
 * No counterpart in the reference: its MLX path has no allocation-free mode. */
h3c_status h3c_attn_fwd_noalloc(const h3c_attn_args* args, void* stream, char* err, size_t err_len);
/* Waits for the current device (cudaDeviceSynchronize), then reads and clears
 * the status word of h3c_attn_fwd_noalloc: H3C_OK, or H3C_ERR_TIMEOUT when a
 * bounded wait of the last call gave up (its output is invalid).  Allocates
 * nothing.  No counterpart in the reference (see h3c_attn_fwd_noalloc). */
h3c_status h3c_attn_fwd_noalloc_status(void);

/* --- sequence-sharded path (NCCL) ------------------------------------------ */
/* Multi-GPU layout for the longest sequences (one process per GPU).  The
 * reference is single-process (batch 1, one device); this is new.  Rank 0
 * creates an id, the caller shares it out of band, every rank initialises its
 * context's communicator (NCCL is loaded at this point with dlopen). */
typedef struct h3c_comm_id {
  char internal[128];
} h3c_comm_id;
h3c_status h3c_comm_unique_id(h3c_comm_id* out);
h3c_status h3c_comm_init(h3c_ctx* ctx, const h3c_comm_id* id, int nranks, int rank);
h3c_status h3c_comm_destroy(h3c_ctx* ctx);   /* also done by h3c_destroy */
/* Each rank passes its token shard: q/k/v/out views of S_r rows, S_r =
 * ceil(ceil(seq_len / nranks) / 128) * 128, shard r holding tokens
 * [r*S_r, (r+1)*S_r); seq_len is the GLOBAL valid length; heads divisible
 * by nranks, head_offset 0, head_count == heads; row_ptr/col_idx and the
 * rope table describe the whole sequence.  Grouped ncclSend/ncclRecv turn
 * [S_r, H, D] into [nranks*S_r, H/nranks, D], the fused call runs on this
 * rank's heads, and the output shard comes back the same way; output rows
 * past seq_len are unspecified.  All work is enqueued on `stream`.  Replaces
 * nothing in the reference (AttentionLayer.sdpa is single-device,
 * Sources/H3Modules/DiTBlock.swift:293-328). */
h3c_status h3c_attn_fwd_seqshard(h3c_ctx* ctx, const h3c_attn_args* args, void* stream);
/* Bounded wait for the work enqueued on `stream` (an h3c_attn_fwd_seqshard
 * call): H3C_OK once it is done; H3C_ERR_NCCL when NCCL reports an error;
 * H3C_ERR_TIMEOUT when it is not done after timeout_ms (a rank that never
 * took part): the communicator is then aborted (its kernels stop), the
 * call's output is invalid and the context's other calls stay usable;
 * h3c_comm_destroy + h3c_comm_init make a new communicator.  The
 * communicator is non-blocking when the process's NCCL supports it (2.14+);
 * with an older NCCL, or with H3C_NCCL_BLOCKING=1 in the environment at
 * h3c_comm_init, a timeout is reported but cannot be aborted.  The
 * non-blocking communicator launches each exchange from NCCL's background
 * thread: measured at 8 B200 on config 2, 18.5 ms per sequence-sharded call
 * against 11.7 ms with a blocking one.
 * Replaces the reference's render-level cancellation
 * (Sources/MiniMaxH3/RenderEngine.swift:574-590) for the exchange. */
h3c_status h3c_comm_wait(h3c_ctx* ctx, void* stream, int64_t timeout_ms);

/* --- synthetic inputs ------------------------------------------------------ */
/* Counter-based N(mean, std) bf16 generator; element i is a function of
 * (seed, stream_id, i) only, bit-identical to the CPU checker's generator. */
h3c_status h3c_fill_normal_bf16(h3c_ctx* ctx, void* d_out, int64_t n, uint64_t seed, uint64_t stream_id,
                                double mean, double std, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* H3CUDA_H */
