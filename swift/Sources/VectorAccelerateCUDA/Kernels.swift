// The reference's kernel classes (Sources/VectorAccelerate/Kernels/Metal4/*.swift) over libva_cuda,
// with their names and high-level signatures. Each holds its context; results follow the
// reference's conventions (uint32 indices, 0xFFFFFFFF padding skipped, squared L2 ascending,
// maximum mode descending, ties by the smaller index).
import CVACuda

private func flatten(_ rows: [[Float]]) throws -> (values: [Float], count: Int, dim: Int) {
    guard let d = rows.first?.count, d > 0 else { throw VectorError.invalidInput("Empty input arrays") }
    guard rows.allSatisfy({ $0.count == d }) else { throw VectorError.invalidInput("Dimension mismatch in input vectors") }
    return (rows.flatMap { $0 }, rows.count, d)
}

/// A resident database (the storage buffer of GPUVectorStorage, Index/Internal/GPUVectorStorage.swift:52-100).
public final class Database: @unchecked Sendable {
    public let context: Metal4Context
    public let handle: OpaquePointer
    public let count: Int
    public let dimension: Int

    public init(context: Metal4Context, vectors: [[Float]], idBase: UInt32 = 0) throws {
        let (flat, n, d) = try flatten(vectors)
        var h: OpaquePointer?
        try flat.withUnsafeBytes {
            try check(va_db_create(context.handle, $0.baseAddress, 0, Int64(n), Int32(d), VA_DTYPE_F32, idBase, &h),
                      "va_db_create")
        }
        try context.synchronize()
        self.context = context
        handle = h!
        count = n
        dimension = d
    }

    /// Row-sharded over a group context (va_db_create_sharded): `vectors` are the rows this
    /// process owns (all rows for `Metal4Context.multi`, this rank's shard for `rank`), `total`
    /// the rows of the whole database.
    public init(sharded context: Metal4Context, vectors: [[Float]], total: Int) throws {
        let (flat, _, d) = try flatten(vectors)
        var h: OpaquePointer?
        try flat.withUnsafeBytes {
            try check(va_db_create_sharded(context.handle, $0.baseAddress, 0, Int64(total), Int32(d), VA_DTYPE_F32, &h),
                      "va_db_create_sharded")
        }
        try context.synchronize()
        self.context = context
        handle = h!
        count = total
        dimension = d
    }

    deinit { va_db_destroy(handle) }

    /// Exact k-NN of host queries (va_knn_search_host): per query up to k (index, distance).
    public func search(queries: [[Float]], k: Int, metric: Int32 = VA_METRIC_L2SQ,
                       precision: Int32 = VA_PREC_AUTO) throws -> [[(index: Int, distance: Float)]] {
        let (flat, nq, d) = try flatten(queries)
        guard d == dimension else { throw VectorError.invalidInput("query dimension \(d) != \(dimension)") }
        var vals = [Float](repeating: 0, count: nq * k)
        var ids = [UInt32](repeating: 0, count: nq * k)
        try flat.withUnsafeBufferPointer { q in
            try vals.withUnsafeMutableBufferPointer { v in
                try ids.withUnsafeMutableBufferPointer { i in
                    try check(va_knn_search_host(context.handle, handle, q.baseAddress, Int64(nq), Int32(k), metric,
                                                 precision, 0, v.baseAddress, i.baseAddress), "va_knn_search_host")
                }
            }
        }
        return (0..<nq).map { r in
            (0..<k).compactMap { j in
                let id = ids[r * k + j]
                return id == 0xFFFF_FFFF ? nil : (index: Int(id), distance: vals[r * k + j])
            }
        }
    }
}

/// FusedL2TopKKernel (Kernels/Metal4/FusedL2TopKKernel.swift:205-1177).
public final class FusedL2TopKKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }

    /// findNearestNeighbors(queries:dataset:k:includeDistances:) (:439-529).
    public func findNearestNeighbors(queries: [[Float]], dataset: [[Float]], k: Int,
                                     includeDistances: Bool = true) async throws -> [[(index: Int, distance: Float)]] {
        guard k > 0 else { throw VectorError.invalidInput("k must be positive") }
        let db = try Database(context: context, vectors: dataset)
        return try db.search(queries: queries, k: k)
    }
}

/// Selection modes (Metal4SelectionMode, TopKSelectionKernel.swift:23-29).
public enum Metal4SelectionMode: Sendable { case minimum, maximum }

/// TopKSelectionKernel (Kernels/Metal4/TopKSelectionKernel.swift:23-519).
public final class TopKSelectionKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }

    /// select(from:k:mode:sorted:) (:369-411): per row the k best (index, value), best first.
    public func select(from values: [[Float]], k: Int, mode: Metal4SelectionMode = .minimum,
                       sorted: Bool = true) async throws -> [[(index: Int, value: Float)]] {
        let (flat, rows, n) = try flatten(values)
        let input = try context.getBuffer(for: flat)
        let ov = try context.getBuffer(size: rows * k * 4)
        let oi = try context.getBuffer(size: rows * k * 4)
        try check(va_topk_select(context.handle, input.pointer.assumingMemoryBound(to: Float.self), Int64(rows),
                                 Int64(n), Int64(n), Int32(k), mode == .minimum ? VA_SELECT_MIN : VA_SELECT_MAX,
                                 ov.pointer.assumingMemoryBound(to: Float.self),
                                 oi.pointer.assumingMemoryBound(to: UInt32.self), Int64(k)), "va_topk_select")
        let v = try ov.download(Float.self, count: rows * k)
        let i = try oi.download(UInt32.self, count: rows * k)
        return (0..<rows).map { r in
            (0..<k).compactMap { j in i[r * k + j] == 0xFFFF_FFFF ? nil : (index: Int(i[r * k + j]), value: v[r * k + j]) }
        }
    }
}

/// All-pairs distance matrices: L2DistanceKernel (L2DistanceKernel.swift:19-89), DotProductKernel
/// (DotProductKernel.swift:25-484) and CosineSimilarityKernel (CosineSimilarityKernel.swift:20-90).
private func matrix(_ context: Metal4Context, _ queries: [[Float]], _ database: [[Float]], metric: Int32,
                    flag: Int32) throws -> [[Float]] {
    let (q, nq, d) = try flatten(queries)
    let (x, nx, dx) = try flatten(database)
    guard d == dx else { throw VectorError.invalidInput("Dimension mismatch in input vectors") }
    let dq = try context.getBuffer(for: q), dxb = try context.getBuffer(for: x)
    let out = try context.getBuffer(size: nq * nx * 4)
    try check(va_distance_matrix(context.handle, dq.pointer.assumingMemoryBound(to: Float.self), Int64(nq),
                                 dxb.pointer.assumingMemoryBound(to: Float.self), Int64(nx), Int32(d), metric, flag,
                                 out.pointer.assumingMemoryBound(to: Float.self), Int64(nx)), "va_distance_matrix")
    let m = try out.download(Float.self, count: nq * nx)
    return (0..<nq).map { Array(m[($0 * nx)..<(($0 + 1) * nx)]) }
}

public final class L2DistanceKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }
    public func distanceMatrix(queries: [[Float]], dataset: [[Float]], computeSqrt: Bool = false) async throws -> [[Float]] {
        try matrix(context, queries, dataset, metric: VA_METRIC_L2SQ, flag: computeSqrt ? 1 : 0)
    }
}

public final class DotProductKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }
    /// compute(queries:database:absoluteValue:) (:365-464).
    public func compute(queries: [[Float]], database: [[Float]], absoluteValue: Bool = false) async throws -> [[Float]] {
        try matrix(context, queries, database, metric: VA_METRIC_IP, flag: absoluteValue ? 1 : 0)
    }
}

public final class CosineSimilarityKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }
    public func distanceMatrix(queries: [[Float]], dataset: [[Float]], outputDistance: Bool = false) async throws -> [[Float]] {
        try matrix(context, queries, dataset, metric: VA_METRIC_COSINE, flag: outputDistance ? 1 : 0)
    }
}

/// ScalarQuantizationKernel (ScalarQuantizationKernel.swift:23-521): global int8 parameters.
public final class ScalarQuantizationKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }

    /// Symmetric int8 quantization (scale = absmax / 127, :496-508) -> (codes, scale).
    public func quantize(_ data: [Float]) async throws -> (codes: [Int8], scale: Float) {
        let absmax = data.reduce(Float(0)) { max($0, abs($1)) }
        let scale = absmax > 0 ? absmax / 127 : 1
        let x = try context.getBuffer(for: data)
        let out = try context.getBuffer(size: max(1, data.count))
        try check(va_sq_quantize_int8(context.handle, x.pointer.assumingMemoryBound(to: Float.self), Int64(data.count),
                                      scale, 0, nil, nil, 0, out.pointer.assumingMemoryBound(to: Int8.self)))
        return (try out.download(Int8.self, count: data.count), scale)
    }

    public func dequantize(_ codes: [Int8], scale: Float) async throws -> [Float] {
        let c = try context.getBuffer(for: codes)
        let out = try context.getBuffer(size: max(1, codes.count * 4))
        try check(va_sq_dequantize_int8(context.handle, c.pointer.assumingMemoryBound(to: Int8.self), Int64(codes.count),
                                        scale, 0, nil, nil, 0, out.pointer.assumingMemoryBound(to: Float.self)))
        return try out.download(Float.self, count: codes.count)
    }
}

/// BinaryQuantizationKernel (BinaryQuantizationKernel.swift:23-513) and HammingDistanceKernel
/// (HammingDistanceKernel.swift:23-609): LSB-first packed codes, Hamming k-NN.
public final class BinaryQuantizationKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }

    /// Packs bit b of word w = (x[32w + b] > 0) per vector -> [n][ceil(d/32)] words.
    public func quantize(vectors: [[Float]]) async throws -> [[UInt32]] {
        let (flat, n, d) = try flatten(vectors)
        let words = (d + 31) / 32
        let x = try context.getBuffer(for: flat)
        let out = try context.getBuffer(size: n * words * 4)
        try check(va_binary_quantize(context.handle, x.pointer.assumingMemoryBound(to: Float.self), Int64(n), Int32(d), 0,
                                     out.pointer.assumingMemoryBound(to: UInt32.self)))
        let w = try out.download(UInt32.self, count: n * words)
        return (0..<n).map { Array(w[($0 * words)..<(($0 + 1) * words)]) }
    }
}

public final class HammingDistanceKernel: @unchecked Sendable {
    public let context: Metal4Context
    public init(context: Metal4Context) { self.context = context }

    /// Fused Hamming k-NN over packed codes: per query up to k (index, distance), (distance, index) order.
    public func nearestNeighbors(queries: [[UInt32]], candidates: [[UInt32]], k: Int) async throws
        -> [[(index: Int, distance: Int)]] {
        guard let words = queries.first?.count, let cw = candidates.first?.count, words == cw else {
            throw VectorError.invalidInput("code widths differ")
        }
        let nq = queries.count, nx = candidates.count
        let q = try context.getBuffer(for: queries.flatMap { $0 }), x = try context.getBuffer(for: candidates.flatMap { $0 })
        let od = try context.getBuffer(size: nq * k * 4), oi = try context.getBuffer(size: nq * k * 4)
        try check(va_hamming_knn(context.handle, q.pointer.assumingMemoryBound(to: UInt32.self), Int64(nq),
                                 x.pointer.assumingMemoryBound(to: UInt32.self), Int64(nx), Int32(words), Int32(k),
                                 od.pointer.assumingMemoryBound(to: UInt32.self),
                                 oi.pointer.assumingMemoryBound(to: UInt32.self)), "va_hamming_knn")
        let d = try od.download(UInt32.self, count: nq * k), i = try oi.download(UInt32.self, count: nq * k)
        return (0..<nq).map { r in
            (0..<k).compactMap { j in i[r * k + j] == 0xFFFF_FFFF ? nil : (index: Int(i[r * k + j]), distance: Int(d[r * k + j])) }
        }
    }
}

// Type aliases of the reference (VectorAccelerate.swift:265-296).
public typealias L2Kernel = L2DistanceKernel
public typealias CosineKernel = CosineSimilarityKernel
public typealias DotKernel = DotProductKernel
public typealias HammingKernel = HammingDistanceKernel
public typealias TopKKernel = TopKSelectionKernel
public typealias FusedTopKKernel = FusedL2TopKKernel
public typealias ScalarQuantKernel = ScalarQuantizationKernel
public typealias BinaryQuantKernel = BinaryQuantizationKernel
