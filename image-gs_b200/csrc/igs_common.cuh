// Shared constants and host-side plumbing of the igs_b200 CUDA library: the compile-time constants of the rasterizer (16x16 tiles, top-10
// lists, normalization epsilon, at most 12 channels; the reference fixes the same values in gsplat/gsplat/cuda/csrc/config.h:1-10), the
// thread-local error message behind igs_last_error(), and launch checking that returns a status instead of exiting the process.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "../../include/igs_b200.h"

namespace igs {

constexpr int kTile = IGS_TILE;                 // pixels per tile side
constexpr int kTilePixels = kTile * kTile;      // one CTA of the tile kernels, one thread per pixel
constexpr int kTopK = IGS_TOP_K;                // Gaussians kept per pixel
constexpr int kMaxChannels = IGS_MAX_CHANNELS;  // feature channels
constexpr double kNormEps = 1e-4;               // added to the sum of the top-K weights (a double in the reference's forward pass)
constexpr uint16_t kNoSlot = 0xFFFF;            // empty entry of the compact per-tile top-K lists

// Record a printf-style message for igs_last_error() and return the status code
int set_error(int status, const char *fmt, ...);

// Status of the last launch on this thread: IGS_OK, or IGS_ERR_CUDA with the CUDA error recorded
int check_launch(const char *what);

inline cudaStream_t as_stream(void *stream) { return reinterpret_cast<cudaStream_t>(stream); }

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

inline bool aligned(const void *p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// sigma of a Gaussian (center gx, gy; conic a, b, c) at a pixel, with the reference's operation order (forward.cu:309-311)
__device__ __forceinline__ float gaussian_sigma(float gx, float gy, float a, float b, float c, float px, float py) {
    // spelled with explicit roundings so that every kernel computes it alike whatever the compiler could share between pixels: the
    // contraction of the reference's fast-math build, 0.5 * fma(a dx, dx, (c dy) dy) fused into fma(b dx, dy, .)
    const float dx = __fsub_rn(gx, px), dy = __fsub_rn(gy, py);
    const float quad = __fmaf_rn(__fmul_rn(a, dx), dx, __fmul_rn(__fmul_rn(c, dy), dy));
    return __fmaf_rn(__fmul_rn(b, dx), dy, __fmul_rn(0.5f, quad));
}

// Programmatic dependent launch (sm_90 and later): the kernels of the training step are launched with programmatic stream serialization,
// and each of them begins with wait_for_predecessor(): griddepcontrol.wait (returns once the predecessor has completed and its writes
// are visible; a no-op for a kernel launched without the attribute) before it reads or writes memory, then
// griddepcontrol.launch_dependents, so that the next kernel on the stream is launched as soon as every CTA of this one has started:
// its CTAs take the SM slots this kernel's finished CTAs free and wait there (in griddepcontrol.wait) for it to complete, instead of
// being launched after it. wait_for_predecessor_only() leaves out the early launch (the peer exchange's kernels).
__device__ __forceinline__ void wait_for_predecessor_only() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void wait_for_predecessor() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace igs

#define IGS_REQUIRE(cond, ...)                                          \
    do {                                                                \
        if (!(cond)) return ::igs::set_error(IGS_ERR_INVALID, __VA_ARGS__); \
    } while (0)
