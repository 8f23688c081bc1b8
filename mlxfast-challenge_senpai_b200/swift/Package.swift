// swift-tools-version:5.9
// SwiftPM package exposing libb2moe (include/b2moe.h) to the Swift runtime:
//   CB2MoE -- system-library C module over the C ABI;
//   B2MoE  -- thin Swift wrappers with the operator signatures the runtime
//             calls (MLX.quantizedMM / gatherQuantizedMM, the MoE block,
//             the expert-parallel prefill), over device pointers and a
//             cudaStream_t.
// Build libb2moe.so first (python mlxfast-challenge_senpai_b200/build.py) and
// point the linker at its directory, e.g.
//   swift build -Xlinker -L<repo>/mlxfast-challenge_senpai_b200/lib \
//               -Xlinker -rpath -Xlinker <repo>/mlxfast-challenge_senpai_b200/lib
import PackageDescription

let package = Package(
    name: "B2MoE",
    products: [
        .library(name: "B2MoE", targets: ["B2MoE"]),
    ],
    targets: [
        .systemLibrary(name: "CB2MoE", path: "Sources/CB2MoE"),
        .target(name: "B2MoE", dependencies: ["CB2MoE"], path: "Sources/B2MoE"),
    ]
)
