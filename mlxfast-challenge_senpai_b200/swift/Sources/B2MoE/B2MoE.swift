// Swift wrappers over the libb2moe C ABI with the signatures of the
// reference runtime's call sites (paths relative to the reference root):
//   MLX.quantizedMM(x, w, scales:, transpose: true, groupSize: 16, bits: 4,
//       mode: .nvfp4)                       Vendor/mlx-swift/Source/MLX/Ops.swift:2433-2453
//   MLX.gatherQuantizedMM(...)              Ops.swift:1468-1488
//   LagunaRuntimeSparseMoEBlock.callAsFunction(x, residual:, routerLogits:)
//                                           Sources/MLXFastModel/LagunaRuntimeModel.swift:9860
// Tensors are device pointers (the CUDA buffers behind evaluated, contiguous,
// row-major arrays) and the stream is a cudaStream_t; turning an MLXArray
// into its device pointer is the runtime's bridge and is not part of this
// package.  Errors surface as B2Error with the library's MLX-style message.
import CB2MoE

public enum B2Error: Error, CustomStringConvertible {
    case failed(code: Int32, message: String)
    public var description: String {
        switch self {
        case let .failed(code, message): return "b2moe error \(code): \(message)"
        }
    }
}

@inline(__always)
func b2check(_ rc: Int32) throws {
    if rc != 0 { throw B2Error.failed(code: rc, message: String(cString: b2_last_error())) }
}

public typealias DevicePointer = UnsafeMutableRawPointer
public typealias CUDAStream = b2_stream_t?

public enum B2DType: Int32 {
    case bf16 = 0, f16 = 1, f32 = 2
}

/// y[M, N] = x[M, K] . dequant(w[N, K/8], scales[N, K/16])^T in x's dtype
/// (drop-in for quantizedMM(..., transpose: true, groupSize: 16, bits: 4,
/// mode: .nvfp4)).
public func quantizedMM(x: DevicePointer, dtype: B2DType, w: DevicePointer, scales: DevicePointer,
                        y: DevicePointer, M: Int, N: Int, K: Int, stream: CUDAStream) throws {
    try b2check(b2_quantized_matmul(x, dtype.rawValue, w.assumingMemoryBound(to: UInt32.self),
                                    scales.assumingMemoryBound(to: UInt8.self), y,
                                    Int64(M), Int64(N), Int64(K), stream))
}

/// y[i] = x[lhs[i]] . W[rhs[i]]^T over P index pairs (drop-in for
/// gatherQuantizedMM in nvfp4 mode).  nil indices mean the identity.
public func gatherQuantizedMM(x: DevicePointer, dtype: B2DType, w: DevicePointer, scales: DevicePointer,
                              lhsIndices: DevicePointer?, rhsIndices: DevicePointer?, pairs: Int,
                              batchX: Int, experts: Int, M: Int, N: Int, K: Int, sortedIndices: Bool,
                              y: DevicePointer, stream: CUDAStream) throws {
    try b2check(b2_gather_qmm(x, dtype.rawValue, w.assumingMemoryBound(to: UInt32.self),
                              scales.assumingMemoryBound(to: UInt8.self),
                              lhsIndices?.assumingMemoryBound(to: UInt32.self),
                              rhsIndices?.assumingMemoryBound(to: UInt32.self), Int64(pairs), Int64(batchX),
                              Int64(experts), Int64(M), Int64(N), Int64(K), sortedIndices ? 1 : 0, y, stream))
}

/// Routed MoE block (router, top-k, SwiGLU experts, ordered combine,
/// residual) -- the routed part of LagunaRuntimeSparseMoEBlock.
public final class B2MoEBlock {
    public var desc = b2_moe_block()

    /// Banks in MLX nvfp4 layout: gate/up [E, F, H/8] + [E, F, H/16], down
    /// [E, H, F/8] + [E, H, F/16]; router weight [E, H] (f32 or bf16).
    /// `decodeBank` / `prefillBank`: buffers of b2_moe_decode_bank_size /
    /// b2_moe_prefill_bank_size bytes to prepare (optional).
    public init(hidden: Int, ffn: Int, experts: Int, topK: Int, laguna: Bool, routerWeight: DevicePointer,
                routerDType: B2DType, routerBias: DevicePointer?, gateCodes: DevicePointer,
                gateScales: DevicePointer, upCodes: DevicePointer, upScales: DevicePointer,
                downCodes: DevicePointer, downScales: DevicePointer, decodeBank: DevicePointer?,
                prefillBank: DevicePointer?, stream: CUDAStream) throws {
        desc.hidden = Int64(hidden)
        desc.ffn = Int64(ffn)
        desc.n_experts = Int64(experts)
        desc.top_k = Int32(topK)
        desc.router_mode = laguna ? Int32(B2_ROUTER_SIGMOID_BIAS) : Int32(B2_ROUTER_SOFTMAX)
        desc.renorm = 1
        desc.routed_scale = laguna ? 2.5 : 1.0
        desc.router_w_dtype = routerDType.rawValue
        desc.router_w = UnsafeRawPointer(routerWeight)
        desc.router_bias = routerBias.map { UnsafePointer($0.assumingMemoryBound(to: Float.self)) }
        desc.gate_codes = UnsafePointer(gateCodes.assumingMemoryBound(to: UInt32.self))
        desc.gate_scales = UnsafePointer(gateScales.assumingMemoryBound(to: UInt8.self))
        desc.up_codes = UnsafePointer(upCodes.assumingMemoryBound(to: UInt32.self))
        desc.up_scales = UnsafePointer(upScales.assumingMemoryBound(to: UInt8.self))
        desc.down_codes = UnsafePointer(downCodes.assumingMemoryBound(to: UInt32.self))
        desc.down_scales = UnsafePointer(downScales.assumingMemoryBound(to: UInt8.self))
        if let bank = decodeBank {
            try b2check(b2_moe_prepare_decode_bank(&desc, bank, b2_moe_decode_bank_size(&desc), stream))
            desc.decode_bank = UnsafeRawPointer(bank)
        }
        if let bank = prefillBank {
            try b2check(b2_moe_prepare_prefill_bank(&desc, bank, b2_moe_prefill_bank_size(&desc), stream))
            desc.prefill_bank = UnsafeRawPointer(bank)
        }
    }

    /// Device scratch bytes a call with `tokens` tokens needs.
    public func workspaceBytes(tokens: Int) -> Int {
        Int(b2_moe_block_workspace_size(&desc, Int64(tokens)))
    }

    /// out = block(x) (+ residual); routerLogits [T, E] f32 replaces the
    /// router GEMV when given.  The workspace (zeroed before its first use)
    /// can be reused by every call on the stream.
    public func callAsFunction(x: DevicePointer, tokens: Int, residual: DevicePointer?, routerLogits: DevicePointer?,
                               out: DevicePointer, workspace: DevicePointer, workspaceBytes: Int,
                               stream: CUDAStream) throws {
        try b2check(b2_moe_block_forward(&desc, x.assumingMemoryBound(to: UInt16.self), Int64(tokens),
                                         routerLogits?.assumingMemoryBound(to: Float.self),
                                         residual?.assumingMemoryBound(to: UInt16.self),
                                         out.assumingMemoryBound(to: UInt16.self), nil, nil, workspace,
                                         workspaceBytes, stream))
    }
}

/// Expert-parallel prefill block: one per process and GPU.  The host moves
/// the handles between ranks (MPI, a TCP store, ...) and calls connect.
public final class B2EPPrefill {
    var ctx: OpaquePointer?
    public private(set) var handle = [UInt8](repeating: 0, count: Int(B2_EP_HANDLE_BYTES))

    /// `block` describes the whole router; its bank pointers hold this
    /// rank's experts only.
    public init(block: B2MoEBlock, rank: Int, world: Int, tokensPerRank: Int, waitTimeoutMs: Int = 10000) throws {
        var cfg = b2_ep_config(rank: Int32(rank), world: Int32(world), tokens_per_rank: Int64(tokensPerRank),
                               wait_timeout_ms: Int32(waitTimeoutMs))
        try handle.withUnsafeMutableBytes { h in
            try b2check(b2_ep_create(&block.desc, &cfg, &ctx, h.baseAddress))
        }
    }

    /// All ranks' handles, concatenated in rank order.
    public func connect(allHandles: [UInt8]) throws {
        try allHandles.withUnsafeBytes { h in try b2check(b2_ep_connect(ctx, h.baseAddress)) }
    }

    public func callAsFunction(x: DevicePointer, tokens: Int, routerLogits: DevicePointer?, residual: DevicePointer?,
                               out: DevicePointer, stream: CUDAStream) throws {
        try b2check(b2_moe_ep_prefill(ctx, x.assumingMemoryBound(to: UInt16.self), Int64(tokens),
                                      routerLogits?.assumingMemoryBound(to: Float.self),
                                      residual?.assumingMemoryBound(to: UInt16.self),
                                      out.assumingMemoryBound(to: UInt16.self), nil, nil, stream))
    }

    deinit { _ = b2_ep_destroy(ctx) }
}
