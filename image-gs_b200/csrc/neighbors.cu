// The k = 8 nearest earlier Gaussians of each Gaussian in bitstream order (causal), or the nearest other ones: the neighbour search of the
// rate model's preparation (compress/rate.py:56-66 bitstream_neighbors -> compress/csrc/prediction.cpp:69-166 nearest_neighbors /
// causal_neighbors), which the reference runs on host threads before each CUDA-graph capture. Integer positions [P, 2]; neighbours ordered
// by squared distance and then by index, -1 where there are fewer. The result is a function of the positions only, so the grid below (any
// cell size gives the same answer) is this file's own.
//
//   1. grid_setup_kernel (one CTA): bounding box, cell size ~ sqrt(2 * area / P) (about two points per cell), doubled until the grid has
//      at most P cells, so the workspace depends on P alone and nothing is read back to the host;
//   2. grid_count_kernel, grid_scan_kernel (one CTA), grid_place_kernel: counting sort of the points by cell;
//   3. neighbors_kernel: one thread per point searches square rings of cells around its own until the next ring cannot hold a nearer
//      point (the ring at Chebyshev cell distance r >= 1 is at least (r - 1) * cell + 1 away), keeping the best eight in registers.
//      Causal queries with at most eight earlier points take all of them directly.
#include "igs_common.cuh"

namespace {

constexpr int kNeighbors = 8;
constexpr int kThreads = 256;
constexpr int kSetupThreads = 1024;

struct GridParams {
    long long min_x, min_y, cell;
    int grid_w, grid_h;
};

struct NeighborWorkspace {
    GridParams params;
    long long pad[10];
    // followed by: int cell_start[max_cells + 1], int cursor[max_cells], int members[P], int cell_of[P]
};

size_t max_cells_of(int num) { return (size_t)(num > 1 ? num : 1); }

size_t workspace_bytes_of(int num) {
    const size_t cells = max_cells_of(num);
    return sizeof(NeighborWorkspace) + sizeof(int) * ((cells + 1) + cells + 2 * (size_t)(num > 0 ? num : 1));
}

__device__ __forceinline__ long long ll_min(long long a, long long b) { return a < b ? a : b; }
__device__ __forceinline__ long long ll_max(long long a, long long b) { return a > b ? a : b; }

__global__ void __launch_bounds__(kSetupThreads) grid_setup_kernel(const int num, const longlong2 *__restrict__ pos, const int max_cells,
                                                                   GridParams *__restrict__ params) {
    __shared__ long long s_red[4][kSetupThreads / 32];
    long long mnx = LLONG_MAX, mny = LLONG_MAX, mxx = LLONG_MIN, mxy = LLONG_MIN;
    for (int i = threadIdx.x; i < num; i += kSetupThreads) {
        const longlong2 p = pos[i];
        mnx = ll_min(mnx, p.x), mny = ll_min(mny, p.y), mxx = ll_max(mxx, p.x), mxy = ll_max(mxy, p.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mnx = ll_min(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
        mny = ll_min(mny, __shfl_xor_sync(0xffffffffu, mny, o));
        mxx = ll_max(mxx, __shfl_xor_sync(0xffffffffu, mxx, o));
        mxy = ll_max(mxy, __shfl_xor_sync(0xffffffffu, mxy, o));
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) s_red[0][warp] = mnx, s_red[1][warp] = mny, s_red[2][warp] = mxx, s_red[3][warp] = mxy;
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < kSetupThreads / 32; ++w) {  // thread 0 holds warp 0's values
        mnx = ll_min(mnx, s_red[0][w]), mny = ll_min(mny, s_red[1][w]);
        mxx = ll_max(mxx, s_red[2][w]), mxy = ll_max(mxy, s_red[3][w]);
    }
    const double area = (double)(mxx - mnx + 1) * (double)(mxy - mny + 1);
    long long cell = (long long)ceil(sqrt(2.0 * area / (double)num));
    cell = cell < 1 ? 1 : cell;
    long long gw = (mxx - mnx) / cell + 1, gh = (mxy - mny) / cell + 1;
    while (gw * gh > max_cells) {
        cell *= 2;
        gw = (mxx - mnx) / cell + 1, gh = (mxy - mny) / cell + 1;
    }
    params->min_x = mnx, params->min_y = mny, params->cell = cell;
    params->grid_w = (int)gw, params->grid_h = (int)gh;
}

__device__ __forceinline__ int cell_index(const longlong2 p, const GridParams &g) {
    return (int)((p.y - g.min_y) / g.cell) * g.grid_w + (int)((p.x - g.min_x) / g.cell);
}

__global__ void grid_count_kernel(const int num, const longlong2 *__restrict__ pos, const GridParams *__restrict__ params,
                                  int *__restrict__ count, int *__restrict__ cell_of) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= num) return;
    const GridParams g = *params;
    const int c = cell_index(pos[i], g);
    cell_of[i] = c;
    atomicAdd(&count[c + 1], 1);
}

// exclusive scan of the counts in place (cell_start[0] = 0 and the counts in cell_start[1..cells]), one CTA, in chunks
__global__ void __launch_bounds__(kSetupThreads) grid_scan_kernel(const GridParams *__restrict__ params, int *__restrict__ cell_start,
                                                                  int *__restrict__ cursor) {
    __shared__ int s_warp[kSetupThreads / 32];
    __shared__ int s_carry;
    const int cells = params->grid_w * params->grid_h;
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 1; base <= cells; base += kSetupThreads) {
        const int idx = base + threadIdx.x;
        int v = idx <= cells ? cell_start[idx] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        if (lane == 31) s_warp[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int w = s_warp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += n;
            }
            s_warp[lane] = w;
        }
        __syncthreads();
        const int incl = v + (warp > 0 ? s_warp[warp - 1] : 0) + s_carry;
        if (idx <= cells) cell_start[idx] = incl;
        __syncthreads();
        if (threadIdx.x == kSetupThreads - 1) s_carry = incl;
        __syncthreads();
    }
    for (int c = threadIdx.x; c < cells; c += kSetupThreads) cursor[c] = cell_start[c];
}

__global__ void grid_place_kernel(const int num, const int *__restrict__ cell_of, int *__restrict__ cursor, int *__restrict__ members) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= num) return;
    members[atomicAdd(&cursor[cell_of[i]], 1)] = i;
}

// best[0..n) sorted by (d2, index); insert (d2, j) if it belongs to the first kNeighbors
__device__ __forceinline__ void offer(long long (&bd)[kNeighbors], int (&bi)[kNeighbors], int &n, const long long d2, const int j) {
    if (n == kNeighbors && !(d2 < bd[kNeighbors - 1] || (d2 == bd[kNeighbors - 1] && j < bi[kNeighbors - 1]))) return;
    long long cd = d2;
    int ci = j;
    // walk from the front: every entry after the candidate's place moves one slot back
#pragma unroll
    for (int k = 0; k < kNeighbors; ++k) {
        if (k >= n + 1) break;
        if (k == n || cd < bd[k] || (cd == bd[k] && ci < bi[k])) {
            const long long td = bd[k];
            const int ti = bi[k];
            bd[k] = cd, bi[k] = ci;
            cd = td, ci = ti;
        }
    }
    n = n < kNeighbors ? n + 1 : n;
}

__global__ void __launch_bounds__(kThreads) neighbors_kernel(const int num, const int causal, const longlong2 *__restrict__ pos,
                                                             const GridParams *__restrict__ params, const int *__restrict__ cell_start,
                                                             const int *__restrict__ members, long long *__restrict__ out_ids,
                                                             long long *__restrict__ out_d2) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= num) return;
    const longlong2 p = pos[i];
    long long bd[kNeighbors];
    int bi[kNeighbors];
    int n = 0;
#pragma unroll
    for (int k = 0; k < kNeighbors; ++k) bd[k] = -1, bi[k] = -1;
    if (causal && i <= kNeighbors) {
        for (int j = 0; j < i; ++j) {
            const longlong2 q = pos[j];
            const long long dx = q.x - p.x, dy = q.y - p.y;
            offer(bd, bi, n, dx * dx + dy * dy, j);
        }
    } else {
        const GridParams g = *params;
        const int cx = (int)((p.x - g.min_x) / g.cell), cy = (int)((p.y - g.min_y) / g.cell);
        const int max_ring = max(max(cx, g.grid_w - 1 - cx), max(cy, g.grid_h - 1 - cy));
        for (int ring = 0; ring <= max_ring; ++ring) {
            if (n == kNeighbors && ring > 0) {
                const long long gap = (long long)(ring - 1) * g.cell + 1;
                if (gap * gap > bd[kNeighbors - 1]) break;
            }
            for (int gy = max(0, cy - ring); gy <= min(g.grid_h - 1, cy + ring); ++gy) {
                const bool edge_row = gy == cy - ring || gy == cy + ring;
                // the square's top and bottom rows are walked cell by cell; a row between them meets the square's border in two
                // cells only, columns cx - ring and cx + ring, so it jumps from one to the other
                const int step = edge_row ? 1 : max(2 * ring, 1);
                for (int gx = cx - ring; gx <= cx + ring; gx += step) {
                    if (gx < 0 || gx >= g.grid_w) continue;
                    const int c = gy * g.grid_w + gx;
                    for (int m = cell_start[c]; m < cell_start[c + 1]; ++m) {
                        const int j = members[m];
                        if (j == i || (causal && j > i)) continue;
                        const longlong2 q = pos[j];
                        const long long dx = q.x - p.x, dy = q.y - p.y;
                        offer(bd, bi, n, dx * dx + dy * dy, j);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kNeighbors; ++k) {
        out_ids[(size_t)i * kNeighbors + k] = k < n ? bi[k] : -1;
        if (out_d2) out_d2[(size_t)i * kNeighbors + k] = k < n ? bd[k] : -1;
    }
}

}  // namespace

extern "C" {

size_t igs_neighbors_workspace(int num_points) { return workspace_bytes_of(num_points); }

int igs_nearest_neighbors(int num_points, const int64_t *positions, int causal, int64_t *neighbors, int64_t *dist2, void *workspace,
                          size_t workspace_bytes, void *stream) {
    IGS_REQUIRE(num_points >= 0, "igs_nearest_neighbors: negative size");
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(positions && neighbors && workspace, "igs_nearest_neighbors: null pointer");
    IGS_REQUIRE(workspace_bytes >= workspace_bytes_of(num_points), "igs_nearest_neighbors: workspace too small (%zu bytes, need %zu)",
                workspace_bytes, workspace_bytes_of(num_points));
    IGS_REQUIRE(igs::aligned(positions, 16) && igs::aligned(workspace, 16), "igs_nearest_neighbors: positions and workspace must be 16-byte aligned");
    cudaStream_t s = igs::as_stream(stream);
    const size_t cells = max_cells_of(num_points);
    NeighborWorkspace *ws = static_cast<NeighborWorkspace *>(workspace);
    int *cell_start = reinterpret_cast<int *>(ws + 1);
    int *cursor = cell_start + cells + 1;
    int *members = cursor + cells;
    int *cell_of = members + num_points;
    const longlong2 *pos = reinterpret_cast<const longlong2 *>(positions);
    if (cudaMemsetAsync(cell_start, 0, sizeof(int) * (cells + 1), s) != cudaSuccess) return igs::check_launch("igs_nearest_neighbors");
    const int blocks = igs::ceil_div(num_points, kThreads);
    grid_setup_kernel<<<1, kSetupThreads, 0, s>>>(num_points, pos, (int)cells, &ws->params);
    grid_count_kernel<<<blocks, kThreads, 0, s>>>(num_points, pos, &ws->params, cell_start, cell_of);
    grid_scan_kernel<<<1, kSetupThreads, 0, s>>>(&ws->params, cell_start, cursor);
    grid_place_kernel<<<blocks, kThreads, 0, s>>>(num_points, cell_of, cursor, members);
    neighbors_kernel<<<blocks, kThreads, 0, s>>>(num_points, causal ? 1 : 0, pos, &ws->params, cell_start, members,
                                                 reinterpret_cast<long long *>(neighbors), reinterpret_cast<long long *>(dist2));
    return igs::check_launch("igs_nearest_neighbors");
}

}  // extern "C"
