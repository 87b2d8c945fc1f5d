// Error reporting and constants of the C ABI (include/igs_b200.h).
#include <cstdarg>
#include <cstdio>

#include "igs_common.cuh"

namespace {
thread_local char g_last_error[1024] = "";
}

namespace igs {

int set_error(int status, const char *fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
    va_end(args);
    return status;
}

int check_launch(const char *what) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return set_error(IGS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    return IGS_OK;
}

}  // namespace igs

extern "C" {

const char *igs_last_error(void) { return g_last_error; }

int igs_version(void) { return IGS_VERSION; }

int igs_constants(int *tile, int *top_k, int *max_channels, double *eps) {
    if (tile) *tile = IGS_TILE;
    if (top_k) *top_k = IGS_TOP_K;
    if (max_channels) *max_channels = IGS_MAX_CHANNELS;
    if (eps) *eps = igs::kNormEps;
    return IGS_OK;
}

}  // extern "C"
