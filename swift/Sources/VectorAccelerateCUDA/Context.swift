// GPUContext over libva_cuda: the CUDA-backed replacement of the reference's Metal4Context
// (Sources/VectorAccelerate/Core/Metal4Context.swift:175-183 init, :342-410 executeAndWait,
// :471-488 getBuffer), keeping its name (VectorAccelerate.swift:254 `GPUContext = Metal4Context`).
import CVACuda

/// Errors of the reference's API (VectorError / IndexError), mapped from the C ABI's status codes.
public enum VectorError: Error, CustomStringConvertible {
    case invalidInput(String)
    case bufferAllocationFailed(String)
    case computeFailed(String)
    case timeout(String)
    case unsupported(String)
    case collectiveFailed(String)

    public var description: String {
        switch self {
        case .invalidInput(let m), .bufferAllocationFailed(let m), .computeFailed(let m), .timeout(let m),
             .unsupported(let m), .collectiveFailed(let m):
            return m
        }
    }
}

/// Throws the error of a non-zero status with the library's thread-local message.
@inline(__always)
func check(_ status: Int32, _ what: String = "") throws {
    if status == VA_OK { return }
    let msg = (va_last_error().map { String(cString: $0) } ?? "") + (what.isEmpty ? "" : " (\(what))")
    switch status {
    case VA_ERR_INVALID_ARG: throw VectorError.invalidInput(msg)
    case VA_ERR_OOM: throw VectorError.bufferAllocationFailed(msg)
    case VA_ERR_TIMEOUT: throw VectorError.timeout(msg)
    case VA_ERR_UNSUPPORTED: throw VectorError.unsupported(msg)
    case VA_ERR_NCCL: throw VectorError.collectiveFailed(msg)
    default: throw VectorError.computeFailed(msg)
    }
}

/// Context options (Metal4Configuration, Core/Metal4Context.swift:13-44).
public struct Metal4Configuration: Sendable {
    public var device: Int32
    public var timeoutMs: UInt32
    public init(device: Int32 = 0, timeoutMs: UInt32 = 120_000) {
        self.device = device
        self.timeoutMs = timeoutMs
    }
}

/// One CUDA device and stream (or, with `multi` / `rank`, a group of devices joined by NCCL).
public final class Metal4Context: @unchecked Sendable {
    public let handle: OpaquePointer
    public let configuration: Metal4Configuration

    public init(configuration: Metal4Configuration = Metal4Configuration()) throws {
        var cfg = va_config(device: configuration.device, timeout_ms: configuration.timeoutMs, stream: nil)
        var h: OpaquePointer?
        try check(va_context_create(&cfg, &h), "va_context_create")
        handle = h!
        self.configuration = configuration
    }

    private init(handle: OpaquePointer, configuration: Metal4Configuration) {
        self.handle = handle
        self.configuration = configuration
    }

    /// All listed devices of this process (va_context_create_multi); searches over a
    /// `ShardedDatabase` then run on every device and merge on devices[0].
    public static func multi(devices: [Int32], timeoutMs: UInt32 = 120_000) throws -> Metal4Context {
        var cfg = va_config(device: devices[0], timeout_ms: timeoutMs, stream: nil)
        var h: OpaquePointer?
        try devices.withUnsafeBufferPointer {
            try check(va_context_create_multi($0.baseAddress, Int32(devices.count), &cfg, &h), "va_context_create_multi")
        }
        return Metal4Context(handle: h!, configuration: Metal4Configuration(device: devices[0], timeoutMs: timeoutMs))
    }

    /// One rank of a group spread over processes (va_context_create_rank); `ncclId` comes from
    /// `Metal4Context.ncclUniqueId()` on one rank.
    public static func rank(_ rank: Int32, of nranks: Int32, ncclId: [UInt8],
                            configuration: Metal4Configuration = Metal4Configuration()) throws -> Metal4Context {
        guard ncclId.count == Int(VA_NCCL_ID_BYTES) else {
            throw VectorError.invalidInput("ncclId must be \(VA_NCCL_ID_BYTES) bytes")
        }
        var cfg = va_config(device: configuration.device, timeout_ms: configuration.timeoutMs, stream: nil)
        var h: OpaquePointer?
        try ncclId.withUnsafeBytes {
            try check(va_context_create_rank(&cfg, nranks, rank, $0.baseAddress, &h), "va_context_create_rank")
        }
        return Metal4Context(handle: h!, configuration: configuration)
    }

    public static func ncclUniqueId() throws -> [UInt8] {
        var id = [UInt8](repeating: 0, count: Int(VA_NCCL_ID_BYTES))
        try id.withUnsafeMutableBytes { try check(va_nccl_unique_id($0.baseAddress), "va_nccl_unique_id") }
        return id
    }

    deinit { va_context_destroy(handle) }

    /// executeAndWait's completion and error check (Metal4Context.swift:377-409): a bounded wait.
    public func synchronize() throws { try check(va_synchronize(handle), "va_synchronize") }

    /// lastGPUTiming (Metal4Context.swift:48-65): device time of the last timed call, in ms.
    public var lastGPUTimeMs: Float {
        var ms: Float = 0
        _ = va_last_gpu_time_ms(handle, &ms)
        return ms
    }

    /// getBuffer(size:) (Metal4Context.swift:471-480).
    public func getBuffer(size: Int) throws -> DeviceBuffer { try DeviceBuffer(context: self, bytes: size) }

    /// getBuffer(for:) (Metal4Context.swift:482-488): a device copy of `values`.
    public func getBuffer<T>(for values: [T]) throws -> DeviceBuffer {
        let b = try DeviceBuffer(context: self, bytes: max(1, values.count * MemoryLayout<T>.stride))
        try b.upload(values)
        return b
    }
}

public typealias GPUContext = Metal4Context
public typealias GPUConfiguration = Metal4Configuration

/// A caller-owned device allocation (MTLBuffer / BufferToken, Core/BufferPool.swift:89-221).
public final class DeviceBuffer: @unchecked Sendable {
    public let context: Metal4Context
    public let bytes: Int
    public let pointer: UnsafeMutableRawPointer

    init(context: Metal4Context, bytes: Int) throws {
        var p: UnsafeMutableRawPointer?
        try check(va_buffer_alloc(context.handle, bytes, &p), "va_buffer_alloc")
        self.context = context
        self.bytes = bytes
        pointer = p!
    }

    deinit { va_buffer_free(context.handle, pointer) }

    public func upload<T>(_ values: [T]) throws {
        let n = values.count * MemoryLayout<T>.stride
        guard n <= bytes else { throw VectorError.invalidInput("upload of \(n) bytes into \(bytes)") }
        try values.withUnsafeBytes { try check(va_buffer_upload(context.handle, pointer, $0.baseAddress, n)) }
        try context.synchronize()
    }

    public func download<T>(_ type: T.Type, count: Int) throws -> [T] where T: Numeric {
        var out = [T](repeating: 0, count: count)
        try out.withUnsafeMutableBytes {
            try check(va_buffer_download(context.handle, $0.baseAddress, pointer, $0.count))
        }
        try context.synchronize()
        return out
    }
}
