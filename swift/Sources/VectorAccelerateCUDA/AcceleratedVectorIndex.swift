// AcceleratedVectorIndex over libva_cuda (flat index): the reference's
// Sources/VectorAccelerate/Index/AcceleratedVectorIndex.swift with its search entry points
// search(query:k:filter:) (:895-934) and search(queries:k:filter:) (:947-1000), stable handles,
// deletion with the fetchK = k + deletedCount over-fetch (:1330) and the iterative filtered search
// (:1188-1265). Rows live in a device database that grows geometrically (va_db_append).
import CVACuda

public struct VectorHandle: Hashable, Sendable {
    public let value: UInt32
}

public typealias VectorMetadata = [String: String]

public struct IndexSearchResult: Sendable {
    public let id: VectorHandle
    public let distance: Float
}

public struct SearchResults: Sendable {
    public var results: [IndexSearchResult] = []
}

public enum SupportedDistanceMetric: Sendable { case euclidean, cosine, dotProduct }

public struct IndexConfiguration: Sendable {
    public var dimension: Int
    public var metric: SupportedDistanceMetric
    public init(dimension: Int, metric: SupportedDistanceMetric = .euclidean) {
        self.dimension = dimension
        self.metric = metric
    }
    public static func flat(dimension: Int, metric: SupportedDistanceMetric = .euclidean) -> IndexConfiguration {
        IndexConfiguration(dimension: dimension, metric: metric)
    }
}

public final class AcceleratedVectorIndex: @unchecked Sendable {
    public let configuration: IndexConfiguration
    public let context: Metal4Context
    private var db: OpaquePointer?
    private var slotHandle: [UInt32] = []
    private var handleSlot: [UInt32: Int] = [:]
    private var deleted: [Bool] = []
    private var metadata: [UInt32: VectorMetadata] = [:]
    private var nextHandle: UInt32 = 0

    public init(configuration: IndexConfiguration, context: Metal4Context? = nil) throws {
        guard configuration.dimension > 0 else { throw VectorError.invalidInput("dimension must be positive") }
        self.configuration = configuration
        self.context = try context ?? Metal4Context()
    }

    deinit { if let db { va_db_destroy(db) } }

    private var metricCode: Int32 {
        switch configuration.metric {
        case .euclidean: return VA_METRIC_L2SQ
        case .cosine: return VA_METRIC_COSINE
        case .dotProduct: return VA_METRIC_IP
        }
    }

    public var count: Int { handleSlot.count }

    /// insert(_:metadata:) (:481-559): appends on the device and returns stable handles.
    @discardableResult
    public func insert(_ vectors: [[Float]], metadata md: [VectorMetadata?]? = nil) throws -> [VectorHandle] {
        guard vectors.allSatisfy({ $0.count == configuration.dimension }) else {
            throw VectorError.invalidInput("dimension mismatch: expected \(configuration.dimension)")
        }
        guard !vectors.isEmpty else { return [] }
        let flat = vectors.flatMap { $0 }
        try flat.withUnsafeBytes { p in
            if let db {
                try check(va_db_append(context.handle, db, p.baseAddress, 0, Int64(vectors.count)), "va_db_append")
            } else {
                var h: OpaquePointer?
                try check(va_db_create(context.handle, p.baseAddress, 0, Int64(vectors.count),
                                       Int32(configuration.dimension), VA_DTYPE_F32, 0, &h), "va_db_create")
                db = h
            }
        }
        var out: [VectorHandle] = []
        for i in 0..<vectors.count {
            let h = nextHandle
            nextHandle += 1
            handleSlot[h] = slotHandle.count
            slotHandle.append(h)
            deleted.append(false)
            if let m = md?[i] { metadata[h] = m }
            out.append(VectorHandle(value: h))
        }
        return out
    }

    /// remove(_:) (:771-798): the slot is masked until compaction.
    public func remove(_ handle: VectorHandle) throws {
        guard let slot = handleSlot.removeValue(forKey: handle.value) else {
            throw VectorError.invalidInput("unknown handle \(handle.value)")
        }
        deleted[slot] = true
        metadata[handle.value] = nil
    }

    /// search(query:k:filter:) (:895-934).
    public func search(query: [Float], k: Int,
                       filter: ((VectorHandle, VectorMetadata?) -> Bool)? = nil) async throws -> SearchResults {
        try await search(queries: [query], k: k, filter: filter)[0]
    }

    /// search(queries:k:filter:) (:947-1000): one device search over the batch, fetching
    /// k + deletedCount (or doubling while a filter rejects candidates), deleted slots dropped.
    public func search(queries: [[Float]], k: Int,
                       filter: ((VectorHandle, VectorMetadata?) -> Bool)? = nil) async throws -> [SearchResults] {
        guard k > 0 else { throw VectorError.invalidInput("k must be positive, got \(k)") }
        guard let db, count > 0 else { return queries.map { _ in SearchResults() } }
        let flat = try queries.map { q -> [Float] in
            guard q.count == configuration.dimension else { throw VectorError.invalidInput("dimension mismatch") }
            return q
        }
        let deletedCount = deleted.lazy.filter { $0 }.count
        var fetch = min(slotHandle.count, filter == nil ? k + deletedCount : 2 * k)
        while true {
            let hits = try fetchNearest(db: db, queries: flat, k: min(fetch, Int(VA_MAX_K)))
            var out: [SearchResults] = []
            var complete = true
            for row in hits {
                var r = SearchResults()
                for (slot, d) in row where !deleted[slot] {
                    let h = VectorHandle(value: slotHandle[slot])
                    if let filter, !filter(h, metadata[h.value]) { continue }
                    r.results.append(IndexSearchResult(id: h, distance: d))
                    if r.results.count == k { break }
                }
                if r.results.count < k && row.count == fetch { complete = false }
                out.append(r)
            }
            let next = min(2 * fetch, slotHandle.count, Int(VA_MAX_K))
            if complete || next == fetch { return out }
            fetch = next
        }
    }

    private func fetchNearest(db: OpaquePointer, queries: [[Float]], k: Int) throws -> [[(Int, Float)]] {
        let nq = queries.count
        let flat = queries.flatMap { $0 }
        var vals = [Float](repeating: 0, count: nq * k)
        var ids = [UInt32](repeating: 0, count: nq * k)
        try flat.withUnsafeBufferPointer { q in
            try vals.withUnsafeMutableBufferPointer { v in
                try ids.withUnsafeMutableBufferPointer { i in
                    try check(va_knn_search_host(context.handle, db, q.baseAddress, Int64(nq), Int32(k), metricCode,
                                                 VA_PREC_AUTO, 0, v.baseAddress, i.baseAddress), "va_knn_search_host")
                }
            }
        }
        return (0..<nq).map { r in
            (0..<k).compactMap { j in ids[r * k + j] == 0xFFFF_FFFF ? nil : (Int(ids[r * k + j]), vals[r * k + j]) }
        }
    }
}
