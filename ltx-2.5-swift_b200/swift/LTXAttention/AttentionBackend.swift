// SPDX-License-Identifier: Apache-2.0
//
// Drop-in body for Sources/LTXAttention/AttentionBackend.swift of
// loading-awesome/LTX-2.5-Swift (today a placeholder, :13-15), binding the C
// ABI of libltxattn_cuda.  Not compiled in this repository: no Swift
// toolchain is available where it was written.  The arguments mirror the SDPA
// switch of DiTAttention.swift:369-382 plus the RoPE of :364-367.
//
// Device buffers are passed as raw CUDA device addresses with [B, H, T, D]
// element strides, so the transposed `split` views (DiTAttention.swift:346-348)
// need no copy.  How an MLXArray exposes its device address depends on the MLX
// backend in use; `DeviceTensor` is the seam for that.

import CLTXAttnCUDA
import Foundation

public enum AttentionBackend {

    /// One [B, H, T, D] device view: address plus element strides (D stride 1).
    public struct DeviceTensor {
        public var address: UnsafeMutableRawPointer
        public var strides: (b: Int64, h: Int64, t: Int64)
        public init(address: UnsafeMutableRawPointer, strides: (b: Int64, h: Int64, t: Int64)) {
            self.address = address
            self.strides = strides
        }
        var c: ltxattn_tensor {
            ltxattn_tensor(data: address, stride_b: strides.b, stride_h: strides.h, stride_t: strides.t)
        }
    }

    /// DiTAttention.Rotary on the device: cos and sin [B, H, T, D/2] in the activation dtype.
    public struct DeviceRotary {
        public var cos: UnsafeRawPointer
        public var sin: UnsafeRawPointer
        public var strides: (b: Int64, h: Int64, t: Int64)
        public var tokens: Int32
        var c: ltxattn_rotary {
            ltxattn_rotary(cos: cos, sin: sin, stride_b: strides.b, stride_h: strides.h,
                           stride_t: strides.t, tokens: tokens)
        }
    }

    /// The `to_gate_logits` output [B, T, heads] on the device (DiTAttention.swift:395-399),
    /// element strides (b, t, h) in the activation dtype.
    public struct DeviceGate {
        public var logits: UnsafeRawPointer
        public var strides: (b: Int64, t: Int64, h: Int64)
        public init(logits: UnsafeRawPointer, strides: (b: Int64, t: Int64, h: Int64)) {
            self.logits = logits
            self.strides = strides
        }
    }

    /// Mirrors DiTAttention.Failure (DiTAttention.swift:107-122) for library errors.
    public struct Failure: Error, CustomStringConvertible {
        public let status: Int32
        public let message: String
        public var description: String { "ltxattn status \(status): \(message)" }
    }

    static func check(_ rc: Int32) throws {
        if rc != 0 { throw Failure(status: rc, message: String(cString: ltxattn_last_error())) }
    }

    /// The fused RoPE + SDPA the `.fused` and `.explicit` arms collapse into.
    /// `keyRotary == nil` with `rotary` given rotates k with `rotary`
    /// (`keyRotary ?? rotary`, DiTAttention.swift:366).  `causal`, `window` and
    /// `kvHeads` give the Gemma encoder's self-attention
    /// (GemmaTextEncoder.swift:218-233, mask :292-323); the DiT passes none.
    /// `gate` fuses the per-head gate `out * 2 * sigmoid(logits)` (DiTAttention.swift:395-399)
    /// into the store; with `out` viewing the merged [B, T, heads * headDim] buffer the
    /// transpose of :401-403 is free as well, so `to_out` reads the result directly.
    public static func attention(
        bf16: Bool, batch: Int32, heads: Int32, queryTokens: Int32, keyTokens: Int32, headDim: Int32,
        q: DeviceTensor, k: DeviceTensor, v: DeviceTensor, out: DeviceTensor, scale: Float,
        keyMask: UnsafePointer<UInt8>? = nil, rotary: DeviceRotary? = nil, keyRotary: DeviceRotary? = nil,
        lse: UnsafeMutablePointer<Float>? = nil, workspace: UnsafeMutableRawPointer?, workspaceBytes: Int,
        causal: Bool = false, window: Int32 = 0, kvHeads: Int32 = 0, gate: DeviceGate? = nil,
        stream: UnsafeMutableRawPointer?
    ) throws {
        var a = ltxattn_fwd_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.heads = heads; a.q_len = queryTokens; a.kv_len = keyTokens; a.head_dim = headDim
        a.q = q.c; a.k = k.c; a.v = v.c; a.out = out.c
        a.scale = scale
        a.key_mask = keyMask
        a.key_mask_stride_b = Int64(keyTokens)
        if let rotary { a.q_rotary = rotary.c }
        if let keyRotary { a.k_rotary = keyRotary.c }
        if let lse {
            a.lse = lse
            a.lse_stride_b = Int64(heads) * Int64(queryTokens)
            a.lse_stride_h = Int64(queryTokens)
        }
        a.workspace = workspace
        a.workspace_bytes = workspaceBytes
        a.causal = causal ? 1 : 0
        a.window = window
        a.kv_heads = kvHeads
        if let gate {
            a.gate = gate.logits
            a.gate_stride_b = gate.strides.b
            a.gate_stride_t = gate.strides.t
            a.gate_stride_h = gate.strides.h
        }
        try check(ltxattn_fwd(&a, stream))
    }

    /// `applySplitRoPE` (DiTAttention.swift:206-234) of one [B, H, T, D] view;
    /// `out` may be `x` itself.
    public static func splitRoPE(
        bf16: Bool, batch: Int32, heads: Int32, tokens: Int32, headDim: Int32,
        x: DeviceTensor, out: DeviceTensor, rotary: DeviceRotary, stream: UnsafeMutableRawPointer?
    ) throws {
        var a = ltxattn_rope_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.heads = heads; a.tokens = tokens; a.head_dim = headDim
        a.x = x.c; a.out = out.c; a.rotary = rotary.c
        try check(ltxattn_rope(&a, stream))
    }

    /// `DiTForward.rotary` (DiTForward.swift:641-678) on the device: per-head tables
    /// [heads, tokens, inner / 2 / heads] from fp32 (lo, hi) positions [nPos, tokens, 2].
    public static func rotaryTables(
        bf16: Bool, positions: UnsafePointer<Float>, nPos: Int32, tokens: Int32, maxPos: [Float],
        inner: Int32, heads: Int32, theta: Double, cos: UnsafeMutableRawPointer, sin: UnsafeMutableRawPointer,
        stream: UnsafeMutableRawPointer?
    ) throws {
        var a = ltxattn_rotary_table_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.n_pos = nPos; a.tokens = tokens; a.inner = inner; a.heads = heads; a.theta = theta
        withUnsafeMutableBytes(of: &a.max_pos) { raw in
            let mp = raw.bindMemory(to: Float.self)
            for (d, v) in maxPos.prefix(4).enumerated() { mp[d] = v }
        }
        a.positions = positions; a.cos = cos; a.sin = sin
        try check(ltxattn_rotary_tables(&a, stream))
    }

    /// The q / k preparation of DiTAttention.swift:358-367 in one pass: rmsNorm over the
    /// inner dim, the head split and split RoPE, from the projection output
    /// [B, tokens, heads * headDim] (element strides `xStrides`) into `out`.
    public static func prepareQK(
        bf16: Bool, batch: Int32, tokens: Int32, heads: Int32, headDim: Int32,
        x: UnsafeRawPointer, xStrides: (b: Int64, t: Int64), weight: UnsafeRawPointer, eps: Float,
        rotary: DeviceRotary?, out: DeviceTensor, stream: UnsafeMutableRawPointer?
    ) throws {
        var a = ltxattn_qk_prep_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.tokens = tokens; a.heads = heads; a.head_dim = headDim
        a.x = x; a.x_stride_b = xStrides.b; a.x_stride_t = xStrides.t
        a.weight = weight; a.eps = eps
        if let rotary { a.rotary = rotary.c }
        a.out = out.c
        try check(ltxattn_qk_prep(&a, stream))
    }

    /// `prepareQK` for q and k in one launch (the key stream may have its own token count);
    /// each result is what `prepareQK` gives for its arguments.
    public static func prepareQKPair(_ q: inout ltxattn_qk_prep_args, _ k: inout ltxattn_qk_prep_args,
                                     stream: UnsafeMutableRawPointer?) throws {
        try check(ltxattn_qk_prep_pair(&q, &k, stream))
    }

    /// Device scratch the same arguments need (call once per shape; the caller allocates).
    public static func workspaceBytes(_ a: inout ltxattn_fwd_args) -> Int {
        Int(ltxattn_fwd_workspace(&a))
    }

    /// What `ltxattn_fwd` will launch for these arguments (for logs and benchmarks).
    public static func plan(_ a: inout ltxattn_fwd_args) throws -> ltxattn_fwd_plan_info {
        var info = ltxattn_fwd_plan_info()
        try check(ltxattn_fwd_plan(&a, &info))
        return info
    }
}
