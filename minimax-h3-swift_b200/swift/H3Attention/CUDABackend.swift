// H3AttentionBackend conformance for the B200 library (libh3cuda, C ABI in
// include/h3cuda.h).  Written against Sources/H3Attention/AttentionBackend.swift
// of MiniMax-H3-Swift; not compile-checked in this repository (no Swift
// toolchain here).

import Foundation
import MLX
import H3Foundation
import H3Hardware
import CH3Cuda

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

    package static func isAvailable(on machine: Machine) -> Bool {
        var n: Int32 = 0
        return h3c_device_count(&n) == H3C_OK && n > 0
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
        if let rowPtr { cudaFreeBridge(rowPtr) }
        if let colIdx { cudaFreeBridge(colIdx) }
        if let ropeTable { cudaFreeBridge(ropeTable) }
        if let ctx { h3c_destroy(ctx) }
    }

    /// Builds the render's block list once (AttentionContext has no geometry).
    package func prepareRender(spec: h3c_mask_spec) throws {
        var s = spec
        var nnz: Int64 = 0
        guard h3c_blockmask_build(&s, nil, nil, 0, &nnz) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 block list", detail: "invalid mask spec")
        }
        let nb = Int((spec.seq_len + spec.block - 1) / spec.block)
        rowPtr = cudaMallocBridge((nb + 1) * 4)
        colIdx = cudaMallocBridge(Int(nnz) * 4)
        guard let ctx, h3c_blockmask_build_device(ctx, &s, rowPtr?.assumingMemoryBound(to: Int32.self),
                                                  colIdx?.assumingMemoryBound(to: Int32.self),
                                                  nnz, &nnz, nil) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 block list", detail: "device build failed")
        }
        seqLen = Int(spec.seq_len)
    }

    /// The render's RoPE table from its packed layout and the checkpoint's
    /// shared `rope.inv_freq` (device fp32, `n` entries): what
    /// `prepareRender` builds in H3Transformer.swift:263-276, for the fused
    /// prologue (H3C_FUSE_PROLOGUE with `a.rope_table` / `a.rope_half`).
    package func prepareRope(layout: h3c_layout_spec, invFreq: UnsafePointer<Float>, n: Int32) throws {
        var spec = layout
        var nseg: Int32 = 0
        var total: Int64 = 0
        var err = [CChar](repeating: 0, count: 256)
        guard h3c_packed_layout(&spec, nil, 0, &nseg, &total, &err, err.count) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 rope table", detail: String(cString: err))
        }
        ropeTable = cudaMallocBridge(Int(total) * Int(3 * n) * 8)
        guard let ctx, h3c_rope_table_layout(ctx, &spec, invFreq, n, ropeTable, total, nil) == H3C_OK else {
            throw H3Error.unavailableFeature(feature: "b200 rope table", detail: "device build failed")
        }
        ropeHalf = 3 * n
    }

    package func attend(queries: MLXArray, keys: MLXArray, values: MLXArray,
                        scale: Float, mask: MLXArray?, context: AttentionContext) -> MLXArray? {
        guard mask == nil, let ctx, let rowPtr, let colIdx,
              queries.ndim == 3, queries.dim(-1) == 128, queries.dim(1) == seqLen,
              context.sequenceLength == seqLen else { return nil }
        let heads = queries.dim(0)
        let out = MLXArray.zeros(queries.shape, dtype: queries.dtype)
        func view(_ a: MLXArray) -> h3c_view {   // [H, S, D]
            h3c_view(ptr: devicePointer(a), token_stride: 128, head_stride: Int64(seqLen * 128))
        }
        var a = h3c_attn_args()
        a.q = view(queries); a.k = view(keys); a.v = view(values); a.out = view(out)
        a.seq_len = Int32(seqLen); a.heads = Int32(heads); a.head_dim = 128
        a.head_offset = 0; a.head_count = Int32(heads)
        a.scale = scale; a.block = 128; a.flags = 0
        a.row_ptr = UnsafePointer(rowPtr.assumingMemoryBound(to: Int32.self))
        a.col_idx = UnsafePointer(colIdx.assumingMemoryBound(to: Int32.self))
        guard h3c_attn_fwd(ctx, &a, currentStream()) == H3C_OK else { return nil }
        return out
    }
}
