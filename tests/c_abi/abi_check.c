/* A plain C caller of the igs_b200 C ABI (no Python, no CUDA headers of its own beyond what igs_b200.h includes): the constants, the
 * workspace sizes, and the host-side argument checks, which return IGS_ERR_INVALID with a message before any GPU work. Built and run by
 * tests/test_cpu_c_abi.py; needs no GPU. Prints one line per check and exits non-zero on the first failure. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "igs_b200.h"

#define CHECK(cond, what)                               \
    do {                                                \
        if (!(cond)) {                                  \
            fprintf(stderr, "FAILED: %s\n", what);      \
            return 1;                                   \
        }                                               \
        printf("ok: %s\n", what);                       \
    } while (0)

int main(void) {
    int tile = 0, top_k = 0, max_c = 0;
    double eps = 0.0;
    CHECK(igs_version() > 0, "igs_version");
    CHECK(igs_constants(&tile, &top_k, &max_c, &eps) == IGS_OK && tile == 16 && top_k == 10 && max_c == 12 && eps == 1e-4,
          "igs_constants: 16x16 tiles, top-10, 12 channels, eps 1e-4");
    CHECK(igs_cumsum_workspace(20000) > 0, "igs_cumsum_workspace");
    CHECK(igs_sort_workspace(356596, 120, 68) >= sizeof(int) * 356596, "igs_sort_workspace");
    CHECK(igs_raster_l1_workspace(8160) >= sizeof(float) * 8160, "igs_raster_l1_workspace");
    CHECK(igs_neighbors_workspace(80000) > 0, "igs_neighbors_workspace");
    CHECK(igs_project_fwd(-1, 0, 0, 0, 8, 8, 1, 1, 0, 0, 0, 0, 0) == IGS_ERR_INVALID && strstr(igs_last_error(), "negative"),
          "igs_project_fwd rejects a negative size");
    CHECK(igs_project_fwd(0, 0, 0, 0, 8, 8, 1, 1, 0, 0, 0, 0, 0) == IGS_OK, "igs_project_fwd accepts zero Gaussians");
    /* a non-null output pointer that is never dereferenced: the channel count is rejected before any use */
    int32_t *fake_topk = (int32_t *)(uintptr_t)256;
    CHECK(igs_raster_fwd_topk(1, 1, 16, 16, 13, 0, 0, 0, 0, 0, 0, fake_topk, 0) == IGS_ERR_INVALID &&
              strstr(igs_last_error(), "channels"),
          "igs_raster_fwd_topk rejects 13 channels");
    CHECK(igs_sort_intersects_noalloc(1, IGS_NOALLOC_MAX_CAPACITY + 1, 0, 0, 0, 1, 1, 0, 0, 0) == IGS_ERR_INVALID,
          "igs_sort_intersects_noalloc rejects a capacity above its scratch");
    return 0;
}
