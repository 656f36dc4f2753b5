// swift-tools-version:5.9
// Swift binding of libva_cuda: the reference's kernel-primitive API (GPUContext, the kernel
// classes, AcceleratedVectorIndex) over the C ABI of include/va_cuda.h. Build on a Linux host with
// a Swift toolchain and the built library:
//   swift build -Xlinker -L<repo>/vectoraccelerate_b200 -Xlinker -rpath -Xlinker <repo>/vectoraccelerate_b200
import PackageDescription

let package = Package(
    name: "VectorAccelerateCUDA",
    products: [
        .library(name: "VectorAccelerateCUDA", targets: ["VectorAccelerateCUDA"]),
    ],
    targets: [
        // The C ABI: a system-library target whose module map exposes va_cuda.h and links va_cuda.
        .systemLibrary(name: "CVACuda", path: "Sources/CVACuda"),
        .target(name: "VectorAccelerateCUDA", dependencies: ["CVACuda"]),
    ]
)
