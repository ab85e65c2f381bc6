// Additions to momij's swift/Package.swift (swift/Package.swift:38-45 declares
// MomijCore): a C target over libmomij_moe.so and a Swift target with the
// SeedlessMetal-shaped shim.  Copy include/momij_moe.h into
// Sources/CMomijMoE/include/ next to module.modulemap, and point the linker
// at the directory that holds libmomij_moe.so (here /opt/momij/lib).
//
// In `targets:` --
        .target(
            name: "CMomijMoE",
            path: "Sources/CMomijMoE",
            linkerSettings: [.unsafeFlags(["-L/opt/momij/lib", "-Xlinker", "-rpath", "-Xlinker", "/opt/momij/lib"])]),
        .target(
            name: "MomijCUDA",
            dependencies: ["CMomijMoE"],
            path: "Sources/MomijCUDA"),
// and add "MomijCUDA" to the dependencies of MomijCore (or of the executable
// that selects the CUDA backend).
