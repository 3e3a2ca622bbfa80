// H3AttentionBackend conformance for the B200 library (libh3cuda, C ABI in
// include/h3cuda.h).  Written against Sources/H3Attention/AttentionBackend.swift
// of MiniMax-H3-Swift; not compile-checked in this repository (no Swift
// toolchain here).

import Foundation
import MLX
import H3Foundation
import H3Hardware
import CH3Cuda

/// What the host's CUDA build of MLX provides to this backend: the device
/// address of an array's buffer and the stream MLX enqueues on.  MLX's Swift
/// API exposes neither, so the host sets `CUDABackend.bridge` once at
/// start-up; without a bridge the backend reports itself unavailable and the
/// registry refuses it (never a silent downgrade).
package protocol H3CUDADeviceBridge: Sendable {
    /// Device pointer of a contiguous, evaluated array (row-major).
    func devicePointer(_ array: MLXArray) -> UnsafeMutableRawPointer?
    /// The cudaStream_t MLX is using on this thread (nil: the default stream).
    func currentStream() -> UnsafeMutableRawPointer?
}

/// Block-sparse attention over a per-render compacted 128x128 block list.
///
/// Declines (returns nil, so the caller runs dense) when no render layout
/// was prepared, when the call's sequence does not match it, or when the
/// geometry is one the kernels refuse (head_dim != 128) -- the decline rule
/// of the reference's fused-prologue fixture.
package final class CUDABackend: H3AttentionBackend, @unchecked Sendable {
    package static let identifier = "b200-block-sparse"
    package static let equivalenceClass: Float = 1e-2
    package static let materialisesScores = false
    package static let prefersMortonOrder = false

    /// Set by the host before the registry resolves a backend.
    nonisolated(unsafe) package static var bridge: H3CUDADeviceBridge?

    package static func isAvailable(on machine: Machine) -> Bool {
        var n: Int32 = 0
        return bridge != nil && h3c_device_count(&n) == H3C_OK && n > 0
    }

    private var ctx: OpaquePointer?
    private var rowPtr: UnsafeMutableRawPointer?
    private var colIdx: UnsafeMutableRawPointer?
    private var seqLen = 0
    private var ropeTable: UnsafeMutableRawPointer?   // bf16 [S, 3n, 4], built once per render
    private var ropeHalf: Int32 = 0

    package required init() {
        var c: OpaquePointer?
        if h3c_init(0, &c) == H3C_OK { ctx = c }
    }

    deinit {
        if let ctx {
            h3c_device_free(ctx, rowPtr)
            h3c_device_free(ctx, colIdx)
            h3c_device_free(ctx, ropeTable)
            h3c_destroy(ctx)
        }
    }

    private func fail(_ feature: String) -> H3Error {
        H3Error.unavailableFeature(feature: feature, detail: ctx.map { String(cString: h3c_last_error($0)) } ?? "no device")
    }

    /// Builds the render's block list once (AttentionContext has no geometry)
    /// into library-owned device memory, and validates it.
    package func prepareRender(spec: h3c_mask_spec) throws {
        guard let ctx else { throw fail("b200 block list") }
        var s = spec
        var nnz: Int64 = 0
        guard h3c_blockmask_build(&s, nil, nil, 0, &nnz) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 block list", detail: "invalid mask spec")
        }
        let nb = Int((spec.seq_len + spec.block - 1) / spec.block)
        h3c_device_free(ctx, rowPtr); rowPtr = nil
        h3c_device_free(ctx, colIdx); colIdx = nil
        guard h3c_device_alloc(ctx, (nb + 1) * 4, &rowPtr) == H3C_OK,
              h3c_device_alloc(ctx, max(Int(nnz), 1) * 4, &colIdx) == H3C_OK,
              h3c_blockmask_build_device(ctx, &s, rowPtr?.assumingMemoryBound(to: Int32.self),
                                         colIdx?.assumingMemoryBound(to: Int32.self), max(nnz, 1), &nnz,
                                         nil) == H3C_OK,
              h3c_blockmask_validate(ctx, rowPtr?.assumingMemoryBound(to: Int32.self),
                                     colIdx?.assumingMemoryBound(to: Int32.self), Int32(nb), nnz, nil) == H3C_OK
        else { throw fail("b200 block list") }
        seqLen = Int(spec.seq_len)
    }

    /// The render's RoPE table from its packed layout and the checkpoint's
    /// shared `rope.inv_freq` (device fp32, `n` entries): what
    /// `prepareRender` builds in H3Transformer.swift:263-276, for the fused
    /// prologue (H3C_FUSE_PROLOGUE with `a.rope_table` / `a.rope_half`).
    package func prepareRope(layout: h3c_layout_spec, invFreq: UnsafePointer<Float>, n: Int32) throws {
        guard let ctx else { throw fail("b200 rope table") }
        var spec = layout
        var nseg: Int32 = 0
        var total: Int64 = 0
        var err = [CChar](repeating: 0, count: 256)
        guard h3c_packed_layout(&spec, nil, 0, &nseg, &total, &err, err.count) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 rope table", detail: String(cString: err))
        }
        h3c_device_free(ctx, ropeTable); ropeTable = nil
        guard h3c_device_alloc(ctx, Int(total) * Int(3 * n) * 8, &ropeTable) == H3C_OK,
              h3c_rope_table_layout(ctx, &spec, invFreq, n, ropeTable, total, nil) == H3C_OK
        else { throw fail("b200 rope table") }
        ropeHalf = 3 * n
    }

    /// Shared by `attend` and `attendFused`: the call's operands as `[H, S, D]`
    /// views, or nil when this call is declined.
    private func args(_ queries: MLXArray, _ keys: MLXArray, _ values: MLXArray, _ out: MLXArray,
                      scale: Float, context: AttentionContext) -> h3c_attn_args? {
        guard let bridge = Self.bridge, rowPtr != nil, colIdx != nil,
              queries.ndim == 3, queries.dim(-1) == 128, queries.dim(1) == seqLen,
              context.sequenceLength == seqLen,
              let qp = bridge.devicePointer(queries), let kp = bridge.devicePointer(keys),
              let vp = bridge.devicePointer(values), let op = bridge.devicePointer(out) else { return nil }
        func view(_ p: UnsafeMutableRawPointer) -> h3c_view {   // [H, S, D]
            h3c_view(ptr: p, token_stride: 128, head_stride: Int64(seqLen * 128))
        }
        var a = h3c_attn_args()
        a.q = view(qp); a.k = view(kp); a.v = view(vp); a.out = view(op)
        a.seq_len = Int32(seqLen); a.heads = Int32(queries.dim(0)); a.head_dim = 128
        a.head_offset = 0; a.head_count = a.heads
        a.scale = scale; a.block = 128; a.flags = 0
        a.row_ptr = UnsafePointer(rowPtr!.assumingMemoryBound(to: Int32.self))
        a.col_idx = UnsafePointer(colIdx!.assumingMemoryBound(to: Int32.self))
        return a
    }

    package func attend(queries: MLXArray, keys: MLXArray, values: MLXArray,
                        scale: Float, mask: MLXArray?, context: AttentionContext) -> MLXArray? {
        guard mask == nil, let ctx else { return nil }
        let out = MLXArray.zeros(queries.shape, dtype: queries.dtype)
        eval(queries, keys, values, out)
        guard var a = args(queries, keys, values, out, scale: scale, context: context),
              h3c_attn_fwd(ctx, &a, Self.bridge?.currentStream()) == H3C_OK else { return nil }
        return out
    }

    /// The fused entry (next to `attend`, as `AttentionLayer.callAsFunction`
    /// would call it, Sources/H3Modules/DiTBlock.swift:346-352): `queries` and
    /// `keys` are the PRE-norm per-head projections; the per-head RMSNorm
    /// (`qNorm`/`kNorm` weights, `eps`, Modulation.swift:116-120) and the
    /// render's split-half RoPE (from `prepareRope`; RMSNorm only when none
    /// was prepared) run inside the call.  Same decline rules as `attend`.
    package func attendFused(queries: MLXArray, keys: MLXArray, values: MLXArray, scale: Float,
                             qNormWeight: MLXArray, kNormWeight: MLXArray, eps: Float,
                             context: AttentionContext) -> MLXArray? {
        guard let ctx, let bridge = Self.bridge, qNormWeight.dim(-1) == 128, kNormWeight.dim(-1) == 128 else {
            return nil
        }
        let out = MLXArray.zeros(queries.shape, dtype: queries.dtype)
        eval(queries, keys, values, out, qNormWeight, kNormWeight)
        guard var a = args(queries, keys, values, out, scale: scale, context: context),
              let wq = bridge.devicePointer(qNormWeight), let wk = bridge.devicePointer(kNormWeight) else {
            return nil
        }
        a.flags = Int32(H3C_FUSE_PROLOGUE.rawValue)
        a.q_norm_weight = UnsafeRawPointer(wq)
        a.k_norm_weight = UnsafeRawPointer(wk)
        a.eps = eps
        if let ropeTable {
            a.rope_table = UnsafeRawPointer(ropeTable)
            a.rope_half = ropeHalf
        } else {
            a.flags |= Int32(H3C_NO_ROPE.rawValue)
        }
        guard h3c_attn_fwd(ctx, &a, bridge.currentStream()) == H3C_OK else { return nil }
        return out
    }
}
