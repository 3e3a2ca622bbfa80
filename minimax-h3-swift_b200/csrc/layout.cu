// Packed-sequence position ids and the production RoPE table, on the device.
//
// The reference builds, once per render, the [S, 3] (t, h, w) position ids
// of the packed sequence text | cond/refs | audio | video in float64
// (PackedLayout.init, Sources/H3Foundation/PackedSequence.swift:192-297, on
// the PositionGrid helpers of :60-147), narrows them to fp32
// (Sources/H3Modules/H3Transformer.swift:270) and turns them into the bf16
// rotation table with the checkpoint's shared inv_freq (:62-78, :271-273).
//
// Here the host walks the segment list once (a few dozen scalars: segment
// bounds, the t origin of each segment, the (origin, step) pairs of the
// area-normalised h and w axes) and the device evaluates every token's
// coordinate from that table, so neither the [S, 3] positions nor the table
// cross PCIe.  Every double operation the reference performs per token is
// repeated in the same order with explicit round-to-nearest intrinsics (no
// contraction into FMA), so the fp32 positions are bit-identical to the
// reference's Float(Double) narrowing.
#include <math.h>
#include <string.h>

#include <vector>

#include "common.cuh"

namespace h3 {
namespace {

constexpr int kMaxSegments = 40;
constexpr double kFrameRescale = 5.0 / 3.0;  // PositionGrid.frameRescale

// How the coordinates of a segment's rows are produced.
enum SegShape : int32_t { kShapeText = 0, kShapeGrid = 1, kShapeAudio = 2 };

struct SegDev {
  int32_t start, stop, shape, frames;  // frames: latent frames of a grid segment; rt of an audio one
  int32_t nh, nw;                      // frame grid (rows of the h and w axes)
  double t0;                           // t origin (grid: first frame; audio: cursor)
  double h_origin, h_step, w_origin, w_step;  // axis value i = (i*step + origin) * 32
  double w_lo, w_hi;                   // audio rows pin w to the axis extremes
};

struct LayoutDev {
  int32_t n_seg;
  int64_t total;
  SegDev seg[kMaxSegments];
};

struct Axis {
  double origin, step;
  int32_t n;
};

// PositionGrid.axis: ratio = dim / sqrt(h*w), n = dim / patch,
// value(i) = (i * (ratio / n) + (1 - ratio) / 2) * 32.
bool make_axis(int dim, int patch, double sqrt_area, Axis* a) {
  double ratio = (double)dim / sqrt_area;
  int n = dim / patch;
  if (n <= 0) return false;
  a->n = n;
  a->step = ratio / (double)n;
  a->origin = (1.0 - ratio) / 2.0;
  return true;
}

__host__ __device__ inline double axis_value(double origin, double step, int32_t i) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(__dadd_rn(__dmul_rn((double)i, step), origin), 32.0);
#else
  volatile double p = (double)i * step;  // keep the host from contracting into an FMA
  volatile double s = p + origin;
  return s * 32.0;
#endif
}

double video_t_span(int n) {
  static const int fpt[5] = {1, 4, 4, 4, 4};
  double acc = 0.0;
  for (int k = 0; k < n; ++k) {
    volatile double inc = kFrameRescale * (double)fpt[k % 5];
    acc = acc + inc;
  }
  return acc;
}

struct Built {
  std::vector<h3c_segment> segments;
  LayoutDev dev;
};

// The segment table of PackedLayout.init; returns an error message or "".
std::string build_layout(const h3c_layout_spec& sp, Built* out) {
  auto& segs = out->segments;
  auto& d = out->dev;
  segs.clear();
  d.n_seg = 0;
  if (sp.text_tokens < 0 || sp.latent_t < 0 || sp.audio_t < 0 || sp.frame_count < 0 || sp.patch <= 0 ||
      sp.n_keyframes < 0 || sp.n_refs < 0 || (sp.n_keyframes && !sp.keyframes) || (sp.n_refs && !sp.refs))
    return "invalid layout spec";
  if ((int64_t)3 + sp.n_keyframes + 2 * (int64_t)sp.n_refs > kMaxSegments)
    return "too many segments (at most " + std::to_string(kMaxSegments) + ")";

  int64_t row = 0;
  auto push = [&](int32_t n, int32_t kind, const SegDev& proto) -> std::string {
    if (row + n > INT32_MAX) return "sequence longer than 2^31-1 tokens";
    SegDev s = proto;
    s.start = (int32_t)row;
    s.stop = (int32_t)(row + n);
    d.seg[d.n_seg++] = s;
    segs.push_back(h3c_segment{s.start, s.stop, kind});
    row += n;
    return "";
  };
  auto grid_proto = [](const Axis& h, const Axis& w, double t0, int frames) {
    SegDev s{};
    s.shape = kShapeGrid;
    s.frames = frames;
    s.nh = h.n;
    s.nw = w.n;
    s.t0 = t0;
    s.h_origin = h.origin; s.h_step = h.step;
    s.w_origin = w.origin; s.w_step = w.step;
    return s;
  };
  auto audio_proto = [](const Axis& w, double t0, int rt) {
    SegDev s{};
    s.shape = kShapeAudio;
    s.frames = rt;
    s.t0 = t0;
    s.w_lo = axis_value(w.origin, w.step, 0);
    s.w_hi = axis_value(w.origin, w.step, w.n - 1);
    return s;
  };

  Axis ha, wa;
  {
    double area = sqrt((double)sp.latent_h * (double)sp.latent_w);
    if (!make_axis(sp.latent_h, sp.patch, area, &ha) || !make_axis(sp.latent_w, sp.patch, area, &wa))
      return "dimension off grid: latent " + std::to_string(sp.latent_w) + "x" + std::to_string(sp.latent_h) +
             " is not a multiple of the patch " + std::to_string(sp.patch);
  }
  std::string e;
  // 1. text: (i, 0, 0)
  SegDev text{};
  text.shape = kShapeText;
  if (!(e = push(sp.text_tokens, H3C_SEG_TEXT, text)).empty()) return e;
  double cursor = (double)sp.text_tokens;
  // 2. keyframes: one frame at PositionGrid.condT
  for (int i = 0; i < sp.n_keyframes; ++i) {
    int p = sp.keyframes[i];
    if (p < 0 || p >= sp.frame_count)
      return "keyframe index " + std::to_string(p) + " is off the timeline of " + std::to_string(sp.frame_count) +
             " frames";
    double ct;
    if (p == 0) ct = (double)sp.text_tokens;
    else if (p == sp.frame_count - 1) {
      volatile double a = (double)sp.text_tokens + video_t_span(sp.latent_t);
      ct = a - kFrameRescale;
    } else {
      volatile double m = kFrameRescale * (double)p;
      ct = (double)sp.text_tokens + m;
    }
    if (!(e = push(ha.n * wa.n, H3C_SEG_COND, grid_proto(ha, wa, ct, 1))).empty()) return e;
  }
  // 3. references
  for (int i = 0; i < sp.n_refs; ++i) {
    const h3c_ref_block& b = sp.refs[i];
    if (b.kind == H3C_REF_IMAGE) {
      Axis rh, rw;
      double area = sqrt((double)b.latent_h * (double)b.latent_w);
      if (!make_axis(b.latent_h, sp.patch, area, &rh) || !make_axis(b.latent_w, sp.patch, area, &rw))
        return "dimension off grid: reference image " + std::to_string(b.latent_w) + "x" + std::to_string(b.latent_h);
      if (!(e = push(rh.n * rw.n, H3C_SEG_REF_IMAGE, grid_proto(rh, rw, cursor, 1))).empty()) return e;
      cursor = cursor + 1.0;
    } else if (b.kind == H3C_REF_AUDIO) {
      if (b.ref_audio_t < 0) return "negative ref_audio_t";
      if (b.ref_audio_t > 0 && !(e = push(2 * b.ref_audio_t, H3C_SEG_REF_AUDIO, audio_proto(wa, cursor, b.ref_audio_t))).empty())
        return e;
      cursor = cursor + (double)b.ref_audio_t;
    } else if (b.kind == H3C_REF_VIDEO || b.kind == H3C_REF_VIDEO_AUDIO) {
      if (b.ref_audio_t < 0 || b.latent_t < 0) return "negative reference length";
      Axis rh, rw;
      double area = sqrt((double)b.latent_h * (double)b.latent_w);
      if (!make_axis(b.latent_h, sp.patch, area, &rh) || !make_axis(b.latent_w, sp.patch, area, &rw))
        return "dimension off grid: reference video " + std::to_string(b.latent_w) + "x" + std::to_string(b.latent_h);
      if (b.ref_audio_t > 0 && !(e = push(2 * b.ref_audio_t, H3C_SEG_REF_AUDIO, audio_proto(rw, cursor, b.ref_audio_t))).empty())
        return e;
      int64_t n = (int64_t)b.latent_t * rh.n * rw.n;
      if (n > INT32_MAX) return "sequence longer than 2^31-1 tokens";
      if (!(e = push((int32_t)n, H3C_SEG_REF_IMAGE, grid_proto(rh, rw, cursor, b.latent_t))).empty()) return e;
      double span = video_t_span(b.latent_t);
      cursor = cursor + ((double)b.ref_audio_t > span ? (double)b.ref_audio_t : span);
    } else {
      return "unknown reference kind " + std::to_string(b.kind);
    }
  }
  // 4. target audio, 5. target video
  if (!(e = push(2 * sp.audio_t, H3C_SEG_AUDIO, audio_proto(wa, cursor, sp.audio_t))).empty()) return e;
  int64_t nv = (int64_t)sp.latent_t * ha.n * wa.n;
  if (nv > INT32_MAX) return "sequence longer than 2^31-1 tokens";
  if (!(e = push((int32_t)nv, H3C_SEG_VIDEO, grid_proto(ha, wa, cursor, sp.latent_t))).empty()) return e;
  d.total = row;
  return "";
}

// Coordinate `axis` (0 t, 1 h, 2 w) of packed row r.
__device__ double position_of(const LayoutDev& L, int64_t r, int axis) {
  int lo = 0;
  while (lo + 1 < L.n_seg && r >= L.seg[lo + 1].start) ++lo;
  const SegDev& s = L.seg[lo];
  const int32_t i = (int32_t)(r - s.start);
  if (s.shape == kShapeText) return axis == 0 ? (double)i : 0.0;
  if (s.shape == kShapeAudio) {
    if (axis == 1) return 0.0;
    const int32_t rt = s.frames;
    if (axis == 2) return i < rt ? s.w_lo : s.w_hi;
    return __dadd_rn(s.t0, (double)(i % rt));
  }
  const int32_t per = s.nh * s.nw;
  const int32_t f = i / per, rem = i - f * per;
  if (axis == 1) return axis_value(s.h_origin, s.h_step, rem / s.nw);
  if (axis == 2) return axis_value(s.w_origin, s.w_step, rem % s.nw);
  // PositionGrid.videoTGrid: origin + the running sum of the frame spans.
  double acc = s.t0;
  for (int k = 0; k < f; ++k) acc = __dadd_rn(acc, __dmul_rn(kFrameRescale, (k % 5) == 0 ? 1.0 : 4.0));
  return acc;
}

__global__ void positions_kernel(LayoutDev L, float* __restrict__ pos) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L.total * 3) return;
  pos[idx] = (float)position_of(L, idx / 3, (int)(idx % 3));
}

// One thread per (token, pair): angle = fp32(pos[axis]) * inv[k], table entry
// (c, -s, s, c) in bf16 (the same arithmetic as rope_table_shared_kernel).
__global__ void rope_layout_kernel(LayoutDev L, const float* __restrict__ inv, int32_t n, uint16_t* __restrict__ table) {
  const int32_t half = 3 * n;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L.total * half) return;
  int64_t s = idx / half;
  int i = (int)(idx % half);
  int axis = i / n;
  float p = (float)position_of(L, s, axis);
  float ang = __fmul_rn(p, inv[i - axis * n]);
  float c = (float)cos((double)ang), sn = (float)sin((double)ang);
  uint16_t* t = table + idx * 4;
  t[0] = f2bf(c);
  t[1] = f2bf(-sn);
  t[2] = f2bf(sn);
  t[3] = f2bf(c);
}

h3c_status fail_layout(h3c_ctx* ctx, h3c_status st, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return st;
}

}  // namespace
}  // namespace h3

extern "C" {

h3c_status h3c_packed_layout(const h3c_layout_spec* spec, h3c_segment* segments, int32_t capacity,
                             int32_t* n_segments, int64_t* total_tokens, char* err, size_t err_len) {
  auto refuse = [&](const std::string& msg) {
    if (err && err_len) {
      const size_t m = msg.size() < err_len - 1 ? msg.size() : err_len - 1;
      memcpy(err, msg.data(), m);
      err[m] = 0;
    }
    return H3C_ERR_INVALID_ARGUMENT;
  };
  if (!spec || !n_segments || !total_tokens || capacity < 0 || (capacity && !segments))
    return refuse("h3c_packed_layout: null or negative argument");
  h3::Built b;
  std::string e = h3::build_layout(*spec, &b);
  if (!e.empty()) return refuse(e);
  *n_segments = (int32_t)b.segments.size();
  *total_tokens = b.dev.total;
  if (capacity && capacity < (int32_t)b.segments.size()) return H3C_ERR_CAPACITY;
  for (size_t i = 0; i < b.segments.size() && (int32_t)i < capacity; ++i) segments[i] = b.segments[i];
  return H3C_OK;
}

h3c_status h3c_packed_positions_device(h3c_ctx* ctx, const h3c_layout_spec* spec, float* d_pos, int64_t capacity,
                                       void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!spec || !d_pos) return h3::fail_layout(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_packed_positions_device: null argument");
  h3::Built b;
  std::string e = h3::build_layout(*spec, &b);
  if (!e.empty()) return h3::fail_layout(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_packed_positions_device: " + e);
  if (capacity < b.dev.total)
    return h3::fail_layout(ctx, H3C_ERR_CAPACITY, "h3c_packed_positions_device: capacity " + std::to_string(capacity) +
                                                      " < " + std::to_string(b.dev.total) + " tokens");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int64_t n = b.dev.total * 3;
  if (n == 0) return H3C_OK;
  h3::positions_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(b.dev, d_pos);
  H3_CUDA_TRY(ctx, cudaGetLastError());
  return H3C_OK;
}

h3c_status h3c_rope_table_layout(h3c_ctx* ctx, const h3c_layout_spec* spec, const float* d_inv_freq, int32_t n,
                                 void* d_table, int64_t capacity, void* stream) {
  if (!ctx) return H3C_ERR_INVALID_ARGUMENT;
  if (!spec || !d_inv_freq || !d_table || n <= 0)
    return h3::fail_layout(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_rope_table_layout: invalid argument");
  if (3 * n > 64) return h3::fail_layout(ctx, H3C_ERR_UNSUPPORTED, "h3c_rope_table_layout: 3*n must be <= 64");
  h3::Built b;
  std::string e = h3::build_layout(*spec, &b);
  if (!e.empty()) return h3::fail_layout(ctx, H3C_ERR_INVALID_ARGUMENT, "h3c_rope_table_layout: " + e);
  if (capacity < b.dev.total)
    return h3::fail_layout(ctx, H3C_ERR_CAPACITY, "h3c_rope_table_layout: capacity " + std::to_string(capacity) + " < " +
                                                      std::to_string(b.dev.total) + " tokens");
  H3_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int64_t total = b.dev.total * 3 * n;
  if (total == 0) return H3C_OK;
  h3::rope_layout_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(b.dev, d_inv_freq, n,
                                                                                           (uint16_t*)d_table);
  H3_CUDA_TRY(ctx, cudaGetLastError());
  return H3C_OK;
}

}  // extern "C"
