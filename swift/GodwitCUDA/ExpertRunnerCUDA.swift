// ExpertRunnerCUDA.swift — the Swift side of the B200 expert path.
//
// Drop-in counterparts, on an HBM-resident expert bank, of the reference
// engine's expert-evaluation entry points:
//   Router.logits / select / route   Sources/Godwit/Runtime/Router.swift:38-104
//   ExpertRunner.apply               Sources/Godwit/Runtime/ExpertRunner.swift:275
//   ExpertRunner.applyBatch          Sources/Godwit/Runtime/ExpertRunner.swift:191-193
//   ExpertRunner.applyAssignments    Sources/Godwit/Runtime/ExpertRunner.swift:108-110
//   the MoE half of TransformerLayer.forward
//                                    Sources/Godwit/Runtime/TransformerLayer.swift:140-238
// Instead of an `ExpertRunner.Weights` buffer (one expert fetched from SSD
// into a slot) the calls name the (layer, expert) of the resident bank; the
// bank is filled once from the bytes ModelReader.loadExpertStride returns.
// Every call goes through include/godwit_cuda.h (module CGodwitCUDA).
import CGodwitCUDA

public struct GodwitCUDAError: Error, CustomStringConvertible {
    public let status: Int32
    public let message: String
    public var description: String { "godwit_cuda status \(status): \(message)" }
}

@inline(__always) func check(_ s: gw_status) throws {
    if s != GW_OK { throw GodwitCUDAError(status: s, message: String(cString: gw_last_error())) }
}

/// One CUDA device's context plus the resident expert bank of a model.
public final class CUDAExpertBank {
    public let hiddenSize: Int
    public let expertCount: Int
    public let topK: Int
    var ctx: OpaquePointer?
    var bank: OpaquePointer?

    /// `expertStride` and the section spans come from the install manifest
    /// (GodwitManifest.expertStride / expertSections); the defaults equal the
    /// reference installer's layout (ExpertLayout, Install/InstallLayout.swift:56-91).
    public init(device: Int32 = 0, hiddenSize: Int, intermediateSize: Int, expertCount: Int,
                layerCount: Int, topK: Int, gptOssActivation: Bool, expertStride: Int? = nil,
                shardRank: Int = 0, shardCount: Int = 1) throws {
        self.hiddenSize = hiddenSize
        self.expertCount = expertCount
        self.topK = topK
        try check(gw_init(device, &ctx))
        var d = gw_bank_desc()
        try check(gw_layout_default(Int32(hiddenSize), Int32(intermediateSize), Int32(expertCount),
                                    Int32(layerCount), Int32(topK),
                                    gptOssActivation ? GW_ACT_GPTOSS_CLAMPED : GW_ACT_SILU, &d))
        if let s = expertStride { d.expert_stride = Int64(s) }
        d.shard_rank = Int32(shardRank)
        d.shard_count = Int32(shardCount)
        try check(gw_bank_create(ctx, &d, &bank))
    }

    deinit {
        if bank != nil { _ = gw_bank_destroy(bank) }
        if ctx != nil { _ = gw_shutdown(ctx) }
    }

    /// The bytes of ModelReader.loadExpertStride (Runtime/ModelReader.swift:73-76)
    /// into HBM; replaces ExpertCache.acquire's slot fill.
    public func upload(layer: Int, expert: Int, stride: UnsafeRawBufferPointer) throws {
        try check(gw_bank_upload_expert(bank, Int32(layer), Int32(expert), stride.baseAddress,
                                        stride.count))
    }

    /// The router's bf16 weight [E, H] and bias [E] (nil: no bias).
    public func uploadRouter(layer: Int, weight: [UInt16], bias: [UInt16]?) throws {
        try weight.withUnsafeBufferPointer { w in
            if let bias = bias {
                try bias.withUnsafeBufferPointer { b in
                    try check(gw_bank_upload_router(bank, Int32(layer), w.baseAddress, b.baseAddress))
                }
            } else {
                try check(gw_bank_upload_router(bank, Int32(layer), w.baseAddress, nil))
            }
        }
    }
}

/// Router.Decision's shape: expert ids highest logit first, softmax over them.
public struct CUDARouterDecision: Equatable {
    public let experts: [Int]
    public let weights: [Float]
}

extension CUDAExpertBank {
    /// Router.logits(for:weight:bias:)
    public func logits(for hidden: [Float16], layer: Int) throws -> [Float] {
        precondition(hidden.count == hiddenSize, "expected \(hiddenSize) inputs")
        var out = [Float](repeating: 0, count: expertCount)
        try hidden.withUnsafeBytes { x in
            try check(gw_router_logits(ctx, bank, Int32(layer), x.baseAddress, GW_DTYPE_F16, 1, &out))
        }
        return out
    }

    /// Router.route(hidden:weight:bias:)
    public func route(hidden: [Float16], layer: Int) throws -> CUDARouterDecision {
        precondition(hidden.count == hiddenSize, "expected \(hiddenSize) inputs")
        var ex = [Int32](repeating: 0, count: topK)
        var wt = [Float](repeating: 0, count: topK)
        try hidden.withUnsafeBytes { x in
            try check(gw_route(ctx, bank, Int32(layer), x.baseAddress, GW_DTYPE_F16, 1, &ex, &wt))
        }
        return CUDARouterDecision(experts: ex.map { Int($0) }, weights: wt)
    }

    /// ExpertRunner.apply(_:weights:): one expert, before the routing weight.
    public func apply(_ input: [Float16], layer: Int, expert: Int) throws -> [Float] {
        precondition(input.count == hiddenSize, "expected \(hiddenSize) inputs")
        var y = [Float](repeating: 0, count: hiddenSize)
        try input.withUnsafeBytes { x in
            try check(gw_expert_apply(ctx, bank, Int32(layer), Int32(expert), x.baseAddress,
                                      GW_DTYPE_F16, &y))
        }
        return y
    }

    /// ExpertRunner.applyBatch(_:experts:): sum of weight * expert(input).
    public func applyBatch(_ input: [Float16], layer: Int,
                           experts: [(expert: Int, weight: Float)]) throws -> [Float] {
        precondition(input.count == hiddenSize, "expected \(hiddenSize) inputs")
        var y = [Float](repeating: 0, count: hiddenSize)
        let ids = experts.map { Int32($0.expert) }
        let ws = experts.map { $0.weight }
        try input.withUnsafeBytes { x in
            try check(gw_expert_apply_batch(ctx, bank, Int32(layer), x.baseAddress, GW_DTYPE_F16,
                                            Int32(experts.count), ids, ws, &y))
        }
        return y
    }

    /// ExpertRunner.applyAssignments for a whole routing decision: inputs
    /// [tokens * H] f16, routing [tokens * topK] (expert, weight) pairs in
    /// rank order; returns [tokens * H] fp32 (the accumulated outputs).
    public func applyAssignments(inputs: [Float16], tokens: Int, layer: Int,
                                 experts: [Int32], weights: [Float]) throws -> [Float] {
        precondition(inputs.count == tokens * hiddenSize && experts.count == tokens * topK
                     && weights.count == experts.count, "inconsistent assignment arrays")
        var out = [Float](repeating: 0, count: tokens * hiddenSize)
        try inputs.withUnsafeBytes { x in
            try check(gw_moe_forward(ctx, bank, Int32(layer), x.baseAddress, GW_DTYPE_F16,
                                     Int32(tokens), experts, weights, &out, nil, nil))
        }
        return out
    }

    /// Route + apply for `tokens` normed rows (the router loop, the demand map
    /// and the ExpertCache + applyAssignments groups of TransformerLayer.forward).
    public func moe(_ normed: [Float16], tokens: Int, layer: Int) throws -> [Float] {
        precondition(normed.count == tokens * hiddenSize, "expected \(tokens * hiddenSize) inputs")
        var out = [Float](repeating: 0, count: normed.count)
        try normed.withUnsafeBytes { x in
            try check(gw_moe_forward(ctx, bank, Int32(layer), x.baseAddress, GW_DTYPE_F16,
                                     Int32(tokens), nil, nil, &out, nil, nil))
        }
        return out
    }

    /// The MoE half of TransformerLayer.forward on the fp32 residual stream:
    /// post-attention RMSNorm, router, experts and `stream += combined`.
    public func moeBlock(_ stream: inout [Float], tokens: Int, layer: Int,
                         postNorm: [UInt16], epsilon: Float) throws {
        precondition(stream.count == tokens * hiddenSize && postNorm.count == hiddenSize,
                     "inconsistent stream or norm sizes")
        try stream.withUnsafeMutableBufferPointer { s in
            try postNorm.withUnsafeBufferPointer { w in
                try check(gw_moe_block(ctx, bank, Int32(layer), s.baseAddress, w.baseAddress,
                                       epsilon, Int32(tokens), nil, nil))
            }
        }
    }
}

/// The trunk's int8 affine projections (Install/Int8Affine.swift format: codes
/// [rows][cols], then a bf16 (scale, zero) pair per row and 64 columns), in
/// place of the Metal int8_affine_gemv / int8_affine_gemv_bias_batched
/// (Sources/Godwit/Metal/MoE/router.metal:65-141) that ModelRunner.project
/// (Runtime/ModelRunner.swift:165-190) and Attention.encodeProjection
/// (Runtime/Attention.swift:218-240) dispatch.  The tensors live on the
/// device (uploaded once, e.g. with cudaMemcpy from the installed trunk.bin
/// section); the calls are ordered on the context's stream.
public final class CUDATrunkProjection {
    let ctx: OpaquePointer?
    public init(context: OpaquePointer?) { ctx = context }

    /// The output head: one f16 token -> fp32 logits [rows].
    public func head(codes: UnsafePointer<UInt8>, meta: UnsafePointer<UInt16>,
                     x: UnsafePointer<UInt16>, rows: Int, cols: Int,
                     y: UnsafeMutablePointer<Float>) throws {
        try check(gw_int8_affine_gemv_async(ctx, codes, meta, nil, x, 1, Int32(rows), Int32(cols),
                                            UnsafeMutableRawPointer(y), GW_DTYPE_F32))
    }

    /// q/k/v/o: `tokens` f16 rows -> f16 [tokens][rows] with the bf16 bias.
    public func project(codes: UnsafePointer<UInt8>, meta: UnsafePointer<UInt16>,
                        bias: UnsafePointer<UInt16>, x: UnsafePointer<UInt16>, tokens: Int,
                        rows: Int, cols: Int, y: UnsafeMutablePointer<UInt16>) throws {
        try check(gw_int8_affine_gemv_async(ctx, codes, meta, bias, x, Int32(tokens), Int32(rows),
                                            Int32(cols), UnsafeMutableRawPointer(y), GW_DTYPE_F16))
    }
}
