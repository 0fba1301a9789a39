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

    /// The VJP of `attention` for LoRA training under gradient checkpointing
    /// (LoRATrainingStep.swift:283-304, GradientCheckpoint.swift:48-67): dq, dk, dv of
    /// sum(dout * out), P recomputed from the forward's `lse` (no stored score matrix).
    /// With rotary tables the gradients are with respect to the un-rotated q and k.
    /// `out` is the forward's un-gated output; `workspace` holds
    /// `backwardWorkspaceBytes` bytes.
    public static func attentionBackward(
        bf16: Bool, batch: Int32, heads: Int32, queryTokens: Int32, keyTokens: Int32, headDim: Int32,
        q: DeviceTensor, k: DeviceTensor, v: DeviceTensor, out: DeviceTensor, dout: DeviceTensor,
        lse: UnsafePointer<Float>, dq: DeviceTensor, dk: DeviceTensor, dv: DeviceTensor, scale: Float,
        keyMask: UnsafePointer<UInt8>? = nil, rotary: DeviceRotary? = nil, keyRotary: DeviceRotary? = nil,
        workspace: UnsafeMutableRawPointer?, workspaceBytes: Int, stream: UnsafeMutableRawPointer?
    ) throws {
        var a = backwardArgs(bf16: bf16, batch: batch, heads: heads, queryTokens: queryTokens,
                             keyTokens: keyTokens, headDim: headDim, q: q, k: k, v: v, out: out, dout: dout,
                             lse: lse, dq: dq, dk: dk, dv: dv, scale: scale, keyMask: keyMask, rotary: rotary,
                             keyRotary: keyRotary)
        a.workspace = workspace
        a.workspace_bytes = workspaceBytes
        try check(ltxattn_bwd(&a, stream))
    }

    /// The argument block of `attentionBackward` (for `backwardWorkspaceBytes`).
    public static func backwardArgs(
        bf16: Bool, batch: Int32, heads: Int32, queryTokens: Int32, keyTokens: Int32, headDim: Int32,
        q: DeviceTensor, k: DeviceTensor, v: DeviceTensor, out: DeviceTensor, dout: DeviceTensor,
        lse: UnsafePointer<Float>, dq: DeviceTensor, dk: DeviceTensor, dv: DeviceTensor, scale: Float,
        keyMask: UnsafePointer<UInt8>? = nil, rotary: DeviceRotary? = nil, keyRotary: DeviceRotary? = nil
    ) -> ltxattn_bwd_args {
        var a = ltxattn_bwd_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.heads = heads; a.q_len = queryTokens; a.kv_len = keyTokens; a.head_dim = headDim
        a.q = q.c; a.k = k.c; a.v = v.c; a.out = out.c; a.dout = dout.c
        a.lse = lse
        a.lse_stride_b = Int64(heads) * Int64(queryTokens)
        a.lse_stride_h = Int64(queryTokens)
        a.dq = dq.c; a.dk = dk.c; a.dv = dv.c
        a.scale = scale
        a.key_mask = keyMask
        a.key_mask_stride_b = Int64(keyTokens)
        if let rotary { a.q_rotary = rotary.c }
        if let keyRotary { a.k_rotary = keyRotary.c }
        return a
    }

    /// Device scratch the backward needs for these arguments (the caller allocates it).
    public static func backwardWorkspaceBytes(_ a: inout ltxattn_bwd_args) -> Int {
        Int(ltxattn_bwd_workspace(&a))
    }

    /// Reads and clears the device's kernel error word (synchronises the device): throws
    /// `Failure` with status LTXATTN_ERR_TIMEOUT when a kernel's bounded wait gave up.
    public static func deviceStatus() throws {
        var site: Int32 = 0
        try check(ltxattn_device_status(1, &site))
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


/// The CUDA device this process renders on, measured rather than assumed: the
/// counterpart of `LTXHardware.Machine` (Machine.swift:31-36), whose fields come from
/// sysctl on a Mac.  Every field here comes from the CUDA runtime through
/// ltxattn_device_query.
public struct CUDAMachine: Equatable {
    public let name: String
    public let device: Int
    public let computeCapability: (major: Int, minor: Int)
    public let smCount: Int
    public let memoryBytes: UInt64
    public let freeBytes: UInt64
    public let l2Bytes: Int
    public let smClockKHz: Int
    /// True when the attention kernels run on this device (sm_100, a B200).
    public let supported: Bool

    public static func == (a: CUDAMachine, b: CUDAMachine) -> Bool {
        a.name == b.name && a.device == b.device && a.computeCapability == b.computeCapability
            && a.smCount == b.smCount && a.memoryBytes == b.memoryBytes && a.l2Bytes == b.l2Bytes
    }

    public var memoryGB: Double { Double(memoryBytes) / 1e9 }

    public static func count() throws -> Int {
        var n: Int32 = 0
        try AttentionBackend.check(ltxattn_device_count(&n))
        return Int(n)
    }

    public static func detect(device: Int = 0) throws -> CUDAMachine {
        var info = ltxattn_device_info()
        try AttentionBackend.check(ltxattn_device_query(Int32(device), &info))
        let name = withUnsafeBytes(of: &info.name) { raw in
            String(decoding: raw.prefix { $0 != 0 }, as: UTF8.self)
        }
        return CUDAMachine(name: name, device: Int(info.device),
                           computeCapability: (Int(info.cc_major), Int(info.cc_minor)),
                           smCount: Int(info.sm_count), memoryBytes: UInt64(info.total_memory_bytes),
                           freeBytes: UInt64(info.free_memory_bytes), l2Bytes: Int(info.l2_bytes),
                           smClockKHz: Int(info.sm_clock_khz), supported: info.supported != 0)
    }

    public var summary: String {
        String(format: "%@ (sm_%d%d), %.0f GB HBM, %d SMs", name, computeCapability.major,
               computeCapability.minor, memoryGB, smCount)
    }
}

/// Whether the attention working set fits the device: the counterpart of
/// `LTXHardware.MemoryPlan` (MemoryPlan.swift:27-34, 62-74).  The reference fits its
/// fused-path activation bytes to MLX allocator peaks (4.67e5 B per video token); here
/// they are the exact buffers of one call (q, k, v, out, lse and the library's
/// workspace; with `training` the backward's too).  `headroomBytes` keeps the
/// reference's meaning: available - peak * (1 + margin).
public struct AttentionMemoryPlan {
    public let info: ltxattn_memory_plan_info
    public var fits: Bool { info.fits != 0 }
    public var peakBytes: Int64 { info.peak_bytes }
    public var headroomBytes: Int64 { info.headroom_bytes }
    public var bytesPerToken: Double { info.bytes_per_token }

    /// `availableBytes == 0` reads the current device's free memory.
    public static func plan(bf16: Bool = true, batch: Int32 = 1, heads: Int32, tokens: Int32, headDim: Int32,
                            rotary: Bool, training: Bool, residentBytes: Int64,
                            availableBytes: Int64 = 0, marginFraction: Double = 0.15) throws -> AttentionMemoryPlan {
        var a = ltxattn_memory_plan_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.heads = heads; a.tokens = tokens; a.head_dim = headDim
        a.rotary = rotary ? 1 : 0
        a.training = training ? 1 : 0
        a.resident_bytes = residentBytes
        a.available_bytes = availableBytes
        a.margin_fraction = marginFraction
        var info = ltxattn_memory_plan_info()
        try AttentionBackend.check(ltxattn_memory_plan(&a, &info))
        return AttentionMemoryPlan(info: info)
    }
}

/// Head-parallel all-gather over NCCL (NVLink / NVSwitch) for a job whose heads are
/// sharded across the GPUs of one box: rank r computes heads [r*H/N, (r+1)*H/N) with
/// `attention(..., head_begin:, head_count:)` and, where a caller needs every head (a
/// non-sharded to_out, DiTAttention.swift:402-404), gathers them.  The reference is
/// single-device; this has no counterpart there.
public final class HeadGather {
    private var comm: OpaquePointer?
    public let ranks: Int
    public let rank: Int

    /// Rank 0 creates the id and shares its 128 bytes with the other ranks out of band.
    public static func uniqueId() throws -> [UInt8] {
        var id = [UInt8](repeating: 0, count: 128)
        try AttentionBackend.check(ltxattn_comm_unique_id(&id))
        return id
    }

    public init(ranks: Int, rank: Int, uniqueId: [UInt8], device: Int) throws {
        precondition(uniqueId.count == 128, "an NCCL unique id is 128 bytes")
        self.ranks = ranks
        self.rank = rank
        var c: OpaquePointer?
        try AttentionBackend.check(ltxattn_comm_init(&c, Int32(ranks), Int32(rank), uniqueId, Int32(device)))
        comm = c
    }

    deinit {
        if let comm { _ = ltxattn_comm_destroy(comm) }
    }

    /// (ranks, rank) as NCCL itself reports them.
    public func size() throws -> (ranks: Int, rank: Int) {
        var n: Int32 = 0, r: Int32 = 0
        try AttentionBackend.check(ltxattn_comm_size(comm, &n, &r))
        return (Int(n), Int(r))
    }

    /// send: contiguous [B, headsPerRank, T, D] on this rank; recv: contiguous
    /// [B, ranks * headsPerRank, T, D] on every rank.
    public func gather(bf16: Bool, batch: Int32, headsPerRank: Int32, tokens: Int32, headDim: Int32,
                       send: UnsafeRawPointer, recv: UnsafeMutableRawPointer,
                       stream: UnsafeMutableRawPointer?) throws {
        var a = ltxattn_gather_args()
        a.dtype = bf16 ? Int32(LTXATTN_BF16.rawValue) : Int32(LTXATTN_F32.rawValue)
        a.batch = batch; a.heads_per_rank = headsPerRank; a.tokens = tokens; a.head_dim = headDim
        a.send = send
        a.recv = recv
        try AttentionBackend.check(ltxattn_allgather_heads(&a, comm, stream))
    }
}
