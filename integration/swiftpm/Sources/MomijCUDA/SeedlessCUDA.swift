// SeedlessCUDA -- the SeedlessMetal entry points of momij's MoE path
// (swift/Sources/MomijCore/SeedlessMetal.swift) over libmomij_moe.so.
// Buffers are device pointers (the caller's CUDA allocations), streams are
// CUDA streams (nil: the default stream, and the call waits for completion,
// like the reference's nil-encoder convention of committing and waiting).
import CMomijMoE

public enum SeedlessCUDAError: Error {
    case unsupportedShape(N: Int, K: Int, gs: Int)
    case notReady
    case noDevice
    case status(Int32)
}

public struct ExpertWeights {
    public var upGateW: UnsafePointer<UInt32>, upGateS: UnsafeRawPointer, upGateB: UnsafeRawPointer
    public var downW: UnsafePointer<UInt32>, downS: UnsafeRawPointer, downB: UnsafeRawPointer
    public init(upGateW: UnsafePointer<UInt32>, upGateS: UnsafeRawPointer, upGateB: UnsafeRawPointer,
                downW: UnsafePointer<UInt32>, downS: UnsafeRawPointer, downB: UnsafeRawPointer) {
        self.upGateW = upGateW; self.upGateS = upGateS; self.upGateB = upGateB
        self.downW = downW; self.downS = downS; self.downB = downB
    }
}

public enum SeedlessCUDA {
    static let bf16 = Int32(MOMIJ_DTYPE_BF16.rawValue)

    static func check(_ rc: Int32, N: Int, K: Int, gs: Int) throws {
        switch rc {
        case 0: return
        case 1: throw SeedlessCUDAError.unsupportedShape(N: N, K: K, gs: gs)
        case 2: throw SeedlessCUDAError.notReady
        case 3: throw SeedlessCUDAError.noDevice
        default: throw SeedlessCUDAError.status(rc)
        }
    }

    public static func workspaceSize(M: Int, Ktop: Int, H: Int, I: Int) -> Int {
        Int(momij_moe_workspace_size(Int32(M), Int32(Ktop), Int32(H), Int32(I)))
    }

    /// SeedlessMetal.gqmm2 (SeedlessMetal.swift:312-438).
    public static func gqmm2(x: UnsafeRawPointer, w: UnsafePointer<UInt32>, scales: UnsafeRawPointer,
                             biases: UnsafeRawPointer, inds: UnsafePointer<Int32>, out: UnsafeMutableRawPointer,
                             Ktop: Int, K: Int, N: Int, gs: Int = 64, lhsPerExpert: Bool = false, M: Int = 1, E: Int,
                             workspace: UnsafeMutableRawPointer, workspaceBytes: Int,
                             stream: UnsafeMutableRawPointer? = nil) throws {
        let rc = momij_moe_gqmm2(x, w, scales, biases, inds, out, Int32(M), Int32(Ktop), Int32(K), Int32(N),
                                 Int32(E), Int32(gs), lhsPerExpert ? 1 : 0, bf16, workspace, workspaceBytes, stream)
        try check(rc, N: N, K: K, gs: gs)
        if stream == nil { try check(momij_moe_synchronize(nil, workspace), N: N, K: K, gs: gs) }
    }

    /// SeedlessMetal.encodeFusedExpert(...residInto:) (SeedlessMetal.swift:503-547) and
    /// SeedlessMoELayer.run (MapleSeedlessMoE.swift:61-77).
    public static func encodeFusedExpert(x: UnsafeRawPointer, weights w: ExpertWeights, inds: UnsafePointer<Int32>,
                                         scores: UnsafePointer<Float>, y: UnsafeMutableRawPointer?,
                                         residInto: UnsafeMutableRawPointer?, H: Int, I: Int, E: Int, Ktop: Int,
                                         gs: Int = 64, M: Int = 1, workspace: UnsafeMutableRawPointer,
                                         workspaceBytes: Int, stream: UnsafeMutableRawPointer? = nil) throws {
        let rc = momij_moe_expert_ffn(x, w.upGateW, w.upGateS, w.upGateB, w.downW, w.downS, w.downB, inds, scores,
                                      y, residInto, Int32(M), Int32(H), Int32(I), Int32(E), Int32(Ktop), Int32(gs),
                                      7.0, bf16, workspace, workspaceBytes, stream)
        try check(rc, N: H, K: I, gs: gs)
        if stream == nil { try check(momij_moe_synchronize(nil, workspace), N: H, K: I, gs: gs) }
    }

    /// SeedlessMetal.encodeMoEBlock (SeedlessMetal.swift:576-609): h += MoE(rmsnorm(h)).
    public static func encodeMoEBlock(h: UnsafeMutableRawPointer, normW: UnsafeRawPointer, gateW: UnsafeRawPointer,
                                      weights w: ExpertWeights, inds: UnsafeMutablePointer<Int32>?,
                                      scores: UnsafeMutablePointer<Float>?, H: Int, I: Int, E: Int, Ktop: Int,
                                      eps: Float, gs: Int = 64, M: Int = 1, workspace: UnsafeMutableRawPointer,
                                      workspaceBytes: Int, stream: UnsafeMutableRawPointer? = nil) throws {
        let rc = momij_moe_block(h, normW, eps, gateW, Int32(MOMIJ_DTYPE_F16.rawValue), w.upGateW, w.upGateS,
                                 w.upGateB, w.downW, w.downS, w.downB, inds, scores, Int32(M), Int32(H), Int32(I),
                                 Int32(E), Int32(Ktop), Int32(gs), 7.0, bf16, workspace, workspaceBytes, stream)
        try check(rc, N: H, K: I, gs: gs)
        if stream == nil { try check(momij_moe_synchronize(nil, workspace), N: H, K: I, gs: gs) }
    }

    /// MapleFused.fusedRouter (MapleFused.swift:79-255); `counter` is the
    /// layer's persistent zeroed uint32 (the reference's routerCtr).
    public static func fusedRouter(x: UnsafeRawPointer, gateW: UnsafeRawPointer, counter: UnsafeMutablePointer<UInt32>,
                                   logitsScratch: UnsafeMutablePointer<Float>, inds: UnsafeMutablePointer<Int32>,
                                   scores: UnsafeMutablePointer<Float>, H: Int, E: Int, topK: Int = 8, M: Int = 1,
                                   stream: UnsafeMutableRawPointer? = nil) throws {
        let rc = momij_moe_fused_router(x, gateW, counter, logitsScratch, inds, scores, Int32(M), Int32(H), Int32(E),
                                        Int32(topK), bf16, Int32(MOMIJ_DTYPE_F16.rawValue), stream)
        try check(rc, N: E, K: H, gs: 0)
    }
}
