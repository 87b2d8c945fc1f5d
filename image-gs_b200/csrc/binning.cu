// Tile binning: the inclusive prefix sum of the tiles hit per Gaussian (compute_cumulative_intersects, gsplat/gsplat/utils.py:96-115) and
// the Gaussian IDs of every tile intersection sorted by tile (sort_intersects_by_tile, gsplat/gsplat/cuda/csrc/bindings.cu:106-167).
//
// The reference maps each intersection slot to its Gaussian by binary search, radix-sorts 32-bit tile keys with CUB (stable, so within a
// tile the Gaussians are in increasing ID order) and finds the tile ranges in a third pass. Here the same order comes from a counting sort
// on the tile grid, with no sort passes over all intersections:
//   1. count:   one thread per intersection slot below min(total, capacity) (the reference drops the slots beyond the capacity, in
//               Gaussian-major order) finds its Gaussian by binary search in the prefix sum and its tile, and takes a rank within the
//               tile from one returning atomic on the tile's counter,
//   2. scan:    one CTA turns the per-tile counts into the tile ranges [start, end) (empty tiles (0, 0)),
//   3. place:   each slot writes its Gaussian at start + rank,
//   4. order:   one warp per tile ranks its few entries (IDs are unique within a tile), restoring increasing Gaussian ID, and zero-fills the
//               padding slots after the last intersection, as the reference's padding entries (key num_tiles, value 0) sort last.
// Every thread does a bounded, balanced amount of work (a large Gaussian's footprint is spread over as many threads as it has tiles).
// Integer-only and deterministic; outputs are bit-identical to the reference for inputs whose tile counts come from the projection.
#include <algorithm>

#include "igs_common.cuh"
#include "igs_internal.cuh"

namespace {

using igs::kTile;

constexpr int kScanThreads = 1024;

// Tile rectangle of a pixel center and integer radius, as the projection computes it (helpers.cuh:11-43 of the reference)
__device__ __forceinline__ void tile_rect(float cx, float cy, float radius, unsigned tiles_x, unsigned tiles_y, unsigned &x0, unsigned &y0,
                                          unsigned &x1, unsigned &y1) {
    const float tcx = cx / (float)kTile, tcy = cy / (float)kTile;
    const float trx = radius / (float)kTile, try_ = radius / (float)kTile;
    x0 = min((unsigned)max(0, (int)(tcx - trx)), tiles_x);
    x1 = min((unsigned)max(0, (int)(tcx + trx + 1)), tiles_x);
    y0 = min((unsigned)max(0, (int)(tcy - try_)), tiles_y);
    y1 = min((unsigned)max(0, (int)(tcy + try_ + 1)), tiles_y);
}

// Inclusive block-wide scan of one value per thread (blockDim.x == kScanThreads); returns the inclusive prefix, *total gets the sum
__device__ __forceinline__ unsigned block_inclusive_scan(unsigned v, unsigned *warp_sums, unsigned *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
        unsigned w = lane < (kScanThreads / 32) ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned n = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += n;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    const unsigned result = v + (warp > 0 ? warp_sums[warp - 1] : 0u);
    *total = warp_sums[kScanThreads / 32 - 1];
    __syncthreads();
    return result;
}

constexpr int kScanItems = 8;  // consecutive elements per thread and chunk: coalesced 32-byte runs

// Scan of in[0, n) by one CTA in chunks of kScanThreads * kScanItems elements; visit(i, exclusive, value) gets each element's exclusive
// prefix (wrapping uint32, as int32 sums). Returns the total.
template <typename Visit>
__device__ __forceinline__ unsigned chunked_scan(const int *__restrict__ in, int n, Visit visit) {
    __shared__ unsigned warp_sums[32];
    unsigned carry = 0u;
    for (int base = 0; base < n; base += kScanThreads * kScanItems) {
        const int first = base + (int)threadIdx.x * kScanItems;
        unsigned v[kScanItems];
        unsigned run = 0u;
        if (first + kScanItems <= n && (reinterpret_cast<uintptr_t>(in + first) & 15) == 0) {
            const int4 a = __ldg(reinterpret_cast<const int4 *>(in + first));
            const int4 b = __ldg(reinterpret_cast<const int4 *>(in + first) + 1);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < kScanItems; ++k) v[k] = first + k < n ? (unsigned)__ldg(&in[first + k]) : 0u;
        }
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) run += v[k];
        unsigned total;
        unsigned excl = block_inclusive_scan(run, warp_sums, &total) - run + carry;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            if (first + k < n) visit(first + k, excl, v[k]);
            excl += v[k];
        }
        carry += total;
    }
    return carry;
}

// Inclusive int32 prefix sum (wrapping, as torch.cumsum in int32) in two fully parallel passes over blocks of kCumBlock elements: the
// block sums, then each block's offset (the sum of the preceding block sums, reduced by the block) and the scan of its own elements
constexpr int kCumThreads = 256;
constexpr int kCumItems = 8;
constexpr int kCumBlock = kCumThreads * kCumItems;

__device__ __forceinline__ void load_items(const int *__restrict__ in, int n, int first, unsigned (&v)[kCumItems]) {
    if (first + kCumItems <= n && (reinterpret_cast<uintptr_t>(in + first) & 15) == 0) {
        const int4 a = __ldg(reinterpret_cast<const int4 *>(in + first));
        const int4 b = __ldg(reinterpret_cast<const int4 *>(in + first) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < kCumItems; ++k) v[k] = first + k < n ? (unsigned)__ldg(&in[first + k]) : 0u;
    }
}

__device__ __forceinline__ unsigned block_sum_u32(unsigned v, unsigned *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    unsigned t = 0u;
#pragma unroll
    for (int w = 0; w < kCumThreads / 32; ++w) t += scratch[w];
    __syncthreads();
    return t;
}

__global__ void __launch_bounds__(kCumThreads) cumsum_partials_kernel(const int n, const int *__restrict__ in, unsigned *__restrict__ partials) {
    igs::wait_for_predecessor();
    __shared__ unsigned scratch[kCumThreads / 32];
    unsigned v[kCumItems], run = 0u;
    load_items(in, n, blockIdx.x * kCumBlock + threadIdx.x * kCumItems, v);
#pragma unroll
    for (int k = 0; k < kCumItems; ++k) run += v[k];
    const unsigned t = block_sum_u32(run, scratch);
    if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// partials: one sum per partials_per_block-th of a block of kCumBlock elements (1: cumsum_partials_kernel's; kCumBlock / 256: the
// training step's projection kernel's sums per 256 Gaussians)
__global__ void __launch_bounds__(kCumThreads) cumsum_scan_kernel(const int n, const int *__restrict__ in, const unsigned *__restrict__ partials,
                                                                  const int partials_per_block, int *__restrict__ out,
                                                                  int *__restrict__ total_out) {
    igs::wait_for_predecessor();
    __shared__ unsigned scratch[kCumThreads / 32];
    unsigned before = 0u;
    for (int b = threadIdx.x; b < (int)blockIdx.x * partials_per_block; b += kCumThreads) before += partials[b];
    before = block_sum_u32(before, scratch);
    const int first = blockIdx.x * kCumBlock + threadIdx.x * kCumItems;
    unsigned v[kCumItems], run = 0u;
    load_items(in, n, first, v);
#pragma unroll
    for (int k = 0; k < kCumItems; ++k) run += v[k];
    // exclusive scan of the per-thread runs within the block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned m = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += m;
    }
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    unsigned warp_before = 0u, block_total = 0u;
#pragma unroll
    for (int w = 0; w < kCumThreads / 32; ++w) {
        warp_before += w < warp ? scratch[w] : 0u;
        block_total += scratch[w];
    }
    unsigned acc = before + warp_before + incl - run;
#pragma unroll
    for (int k = 0; k < kCumItems; ++k) {
        acc += v[k];
        if (first + k < n) out[first + k] = (int)acc;
    }
    if (total_out && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) *total_out = (int)(before + block_total);
}

// Tile key of slot `local` of a Gaussian's footprint: row-major position in its tile rectangle (forward.cu:102-103 of the reference)
__device__ __forceinline__ unsigned slot_tile(int local, unsigned x0, unsigned y0, unsigned width, unsigned tiles_x) {
    return (y0 + (unsigned)local / width) * tiles_x + x0 + (unsigned)local % width;
}

// The Gaussian owning intersection slot idx: the first g with cum[g] > idx (forward.cu:89-98 of the reference)
__device__ __forceinline__ int owner_of(const int *__restrict__ cum, int n, int idx) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(&cum[mid]) > idx)
            hi = mid;
        else
            lo = mid + 1;
    }
    return lo;
}

// One thread per intersection slot below min(total, capacity): its Gaussian, its tile, and a rank within the tile from the returning
// atomic on the tile's counter (arbitrary order; the order pass restores increasing Gaussian ID). Only the tile rows [row_begin, row_end)
// are binned (a band of the image; the whole grid otherwise): each Gaussian's rectangle is clipped to them, tiles are numbered within the
// band, and the prefix sum must count the clipped rectangles (igs_band_tiles_hit).
__global__ void __launch_bounds__(256) count_kernel(const int n, const int capacity, const float2 *__restrict__ xys,
                                                    const int *__restrict__ radii, const int *__restrict__ cum, const unsigned tiles_x,
                                                    const unsigned tiles_y, const unsigned row_begin, const unsigned row_end,
                                                    int *__restrict__ tile_count, int2 *__restrict__ slot_tile_rank,
                                                    int *__restrict__ slot_gaussian) {
    igs::wait_for_predecessor();
    const int slots = min(__ldg(&cum[n - 1]), capacity);
    const unsigned num_tiles = tiles_x * (row_end - row_begin);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < slots; idx += gridDim.x * blockDim.x) {
        const int g = owner_of(cum, n, idx);
        const int local = idx - (g > 0 ? __ldg(&cum[g - 1]) : 0);
        const float2 xy = __ldg(&xys[g]);
        unsigned x0, y0, x1, y1;
        tile_rect(xy.x, xy.y, (float)__ldg(&radii[g]), tiles_x, tiles_y, x0, y0, x1, y1);
        y0 = max(y0, row_begin);
        y1 = min(y1, row_end);
        const unsigned width = x1 - x0;
        unsigned tile = num_tiles;  // inconsistent inputs (an empty footprint with slots): dropped
        if (width > 0 && y1 > y0) tile = slot_tile(local, x0, y0 - row_begin, width, tiles_x);
        int rank = -1;
        if (tile < num_tiles) rank = atomicAdd(&tile_count[tile], 1);
        slot_tile_rank[idx] = make_int2((int)tile, rank);
        slot_gaussian[idx] = g;
    }
}

// Tiles of the rows [row_begin, row_end) that each Gaussian's rectangle covers (the band's num_tiles_hit)
__global__ void __launch_bounds__(256) band_hits_kernel(const int n, const float2 *__restrict__ xys, const int *__restrict__ radii,
                                                        const unsigned tiles_x, const unsigned tiles_y, const unsigned row_begin,
                                                        const unsigned row_end, int *__restrict__ hits) {
    igs::wait_for_predecessor();
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    int count = 0;
    const int radius = __ldg(&radii[g]);
    if (radius > 0) {
        const float2 xy = __ldg(&xys[g]);
        unsigned x0, y0, x1, y1;
        tile_rect(xy.x, xy.y, (float)radius, tiles_x, tiles_y, x0, y0, x1, y1);
        y0 = max(y0, row_begin);
        y1 = min(y1, row_end);
        if (y1 > y0) count = (int)((x1 - x0) * (y1 - y0));
    }
    hits[g] = count;
}

// Exclusive scan of the tile counts by one CTA: tile_bins[t] = (start, end), (0, 0) for empty tiles
__global__ void __launch_bounds__(kScanThreads) tile_scan_kernel(const int num_tiles, const int *__restrict__ tile_count,
                                                                 int2 *__restrict__ tile_bins, int *__restrict__ total_out) {
    igs::wait_for_predecessor();
    const unsigned total = chunked_scan(tile_count, num_tiles, [&](int t, unsigned excl, unsigned v) {
        tile_bins[t] = v > 0u ? make_int2((int)excl, (int)(excl + v)) : make_int2(0, 0);
    });
    if (threadIdx.x == 0) *total_out = (int)total;
}

// Each slot's Gaussian to its tile's range at its rank
__global__ void __launch_bounds__(256) place_kernel(const int n, const int capacity, const int *__restrict__ cum, const unsigned num_tiles,
                                                    const int2 *__restrict__ tile_bins, const int2 *__restrict__ slot_tile_rank,
                                                    const int *__restrict__ slot_gaussian, int *__restrict__ unsorted) {
    igs::wait_for_predecessor();
    const int slots = min(__ldg(&cum[n - 1]), capacity);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < slots; idx += gridDim.x * blockDim.x) {
        const int2 tr = slot_tile_rank[idx];
        if ((unsigned)tr.x < num_tiles) unsorted[tile_bins[tr.x].x + tr.y] = slot_gaussian[idx];
    }
}

constexpr int kOrderWarps = 8;
constexpr int kOrderStage = 1024;  // entries per warp staged in shared memory

// One warp per tile: each entry's final position is the number of smaller IDs in its tile (IDs are unique within a tile). Lists up to 32
// entries stay in registers, up to kOrderStage in shared memory, longer ones are ranked from global memory. Also zero-fills the padding
// slots [total, capacity).
__global__ void __launch_bounds__(kOrderWarps * 32) order_kernel(const int num_tiles, const int capacity, const int2 *__restrict__ tile_bins,
                                                                 const int *__restrict__ unsorted, const int *__restrict__ total_in,
                                                                 int *__restrict__ sorted) {
    igs::wait_for_predecessor();
    __shared__ int stage[kOrderWarps][kOrderStage];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tile = blockIdx.x * kOrderWarps + warp;

    // padding after the last intersection
    const int total = min(*total_in, capacity);
    for (int i = total + blockIdx.x * blockDim.x + threadIdx.x; i < capacity; i += gridDim.x * blockDim.x) sorted[i] = 0;

    if (tile >= num_tiles) return;
    const int2 range = tile_bins[tile];
    const int len = range.y - range.x;
    if (len <= 0) return;
    const int *src = unsorted + range.x;
    int *dst = sorted + range.x;
    if (len <= 32) {
        const int v = lane < len ? src[lane] : INT_MAX;
        int rank = 0;
        for (int j = 0; j < len; ++j) rank += __shfl_sync(0xffffffffu, v, j) < v;
        if (lane < len) dst[rank] = v;
    } else if (len <= kOrderStage) {
        int *buf = stage[warp];
        for (int j = lane; j < len; j += 32) buf[j] = src[j];
        __syncwarp();
        for (int e = lane; e < len; e += 32) {
            const int v = buf[e];
            int rank = 0;
            for (int j = 0; j < len; ++j) rank += buf[j] < v;
            dst[rank] = v;
        }
    } else {
        for (int e = lane; e < len; e += 32) {
            const int v = src[e];
            int rank = 0;
            for (int j = 0; j < len; ++j) rank += __ldg(&src[j]) < v;
            dst[rank] = v;
        }
    }
}

size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t sort_workspace_bytes(int capacity, int num_tiles) {
    // tile counts, the intersection total, per-slot (tile, rank) and Gaussian, and the unsorted IDs
    const size_t cap = capacity > 0 ? (size_t)capacity : 0;
    return round256(sizeof(int) * (size_t)num_tiles) + round256(sizeof(int)) + round256(sizeof(int2) * cap) + 2 * round256(sizeof(int) * cap);
}

}  // namespace

extern "C" {

size_t igs_cumsum_workspace(int n) { return sizeof(unsigned) * (size_t)igs::ceil_div(n > 0 ? n : 1, kCumBlock); }

int igs_cumsum(int n, const int32_t *num_tiles_hit, int32_t *cum_tiles_hit, int32_t *total, void *workspace, size_t workspace_bytes,
               void *stream) {
    IGS_REQUIRE(n >= 0, "igs_cumsum: negative size");
    cudaStream_t s = igs::as_stream(stream);
    if (n == 0) {
        if (total && cudaMemsetAsync(total, 0, sizeof(int), s) != cudaSuccess) return igs::check_launch("igs_cumsum");
        return IGS_OK;
    }
    IGS_REQUIRE(num_tiles_hit && cum_tiles_hit && workspace, "igs_cumsum: null pointer");
    IGS_REQUIRE(workspace_bytes >= igs_cumsum_workspace(n), "igs_cumsum: workspace too small");
    const int blocks = igs::ceil_div(n, kCumBlock);
    unsigned *partials = static_cast<unsigned *>(workspace);
    igs::launch(cumsum_partials_kernel, blocks, kCumThreads, 0, s, n, num_tiles_hit, partials);
    igs::launch(cumsum_scan_kernel, blocks, kCumThreads, 0, s, n, num_tiles_hit, partials, 1, cum_tiles_hit, total);
    return igs::check_launch("igs_cumsum");
}

size_t igs_sort_workspace(int capacity, int tiles_x, int tiles_y) { return sort_workspace_bytes(capacity, tiles_x * tiles_y); }

static int sort_band(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit, int tiles_x,
                     int tiles_y, int row_begin, int row_end, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *workspace,
                     size_t workspace_bytes, void *stream, const char *who, bool counters_zeroed = false) {
    IGS_REQUIRE(num_points >= 0 && tiles_x >= 0 && tiles_y >= 0, "%s: negative size", who);
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "%s: tile rows [%d, %d) outside [0, %d)", who, row_begin,
                row_end, tiles_y);
    const int num_tiles = tiles_x * (row_end - row_begin);
    cudaStream_t s = igs::as_stream(stream);
    if (num_tiles == 0) return IGS_OK;
    IGS_REQUIRE(tile_bins != nullptr, "%s: null tile_bins", who);
    IGS_REQUIRE(igs::aligned(tile_bins, 8), "%s: tile_bins must be 8-byte aligned [T, 2] int32", who);
    if (capacity <= 0) {
        // the reference returns no intersections and zero tile ranges (bindings.cu:124-126)
        if (cudaMemsetAsync(tile_bins, 0, sizeof(int) * 2 * (size_t)num_tiles, s) != cudaSuccess) return igs::check_launch(who);
        return IGS_OK;
    }
    IGS_REQUIRE(gaussian_ids_sorted && workspace, "%s: null pointer", who);
    IGS_REQUIRE(workspace_bytes >= sort_workspace_bytes(capacity, num_tiles), "%s: workspace too small (%zu < %zu)", who, workspace_bytes,
                sort_workspace_bytes(capacity, num_tiles));
    IGS_REQUIRE(num_points == 0 || (xys && radii && cum_tiles_hit), "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || igs::aligned(xys, 8), "%s: xys must be 8-byte aligned", who);

    char *ws = static_cast<char *>(workspace);
    int *tile_count = reinterpret_cast<int *>(ws);
    ws += round256(sizeof(int) * (size_t)num_tiles);
    int *total = reinterpret_cast<int *>(ws);
    ws += round256(sizeof(int));
    int2 *slot_tile_rank = reinterpret_cast<int2 *>(ws);
    ws += round256(sizeof(int2) * (size_t)capacity);
    int *slot_gaussian = reinterpret_cast<int *>(ws);
    ws += round256(sizeof(int) * (size_t)capacity);
    int *unsorted = reinterpret_cast<int *>(ws);

    if (!counters_zeroed && cudaMemsetAsync(tile_count, 0, sizeof(int) * (size_t)num_tiles, s) != cudaSuccess) return igs::check_launch(who);
    // slots are bounded by the capacity; a grid-stride loop over them reads the true count on the device
    const int slot_blocks = std::min(igs::ceil_div(capacity, 256), 148 * 16);
    if (num_points > 0) {
        igs::launch(count_kernel, slot_blocks, 256, 0, s, num_points, capacity, reinterpret_cast<const float2 *>(xys), radii,
                    cum_tiles_hit, (unsigned)tiles_x, (unsigned)tiles_y, (unsigned)row_begin, (unsigned)row_end, tile_count, slot_tile_rank,
                    slot_gaussian);
    }
    igs::launch(tile_scan_kernel, 1, kScanThreads, 0, s, num_tiles, tile_count, reinterpret_cast<int2 *>(tile_bins), total);
    if (num_points > 0) {
        igs::launch(place_kernel, slot_blocks, 256, 0, s, num_points, capacity, cum_tiles_hit, (unsigned)num_tiles,
                    reinterpret_cast<const int2 *>(tile_bins), slot_tile_rank, slot_gaussian, unsorted);
    }
    igs::launch(order_kernel, igs::ceil_div(num_tiles, kOrderWarps), kOrderWarps * 32, 0, s, num_tiles, capacity,
                reinterpret_cast<const int2 *>(tile_bins), unsorted, total, gaussian_ids_sorted);
    return igs::check_launch(who);
}

int igs_sort_intersects(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit, int tiles_x,
                        int tiles_y, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *workspace, size_t workspace_bytes,
                        void *stream) {
    return sort_band(num_points, capacity, xys, radii, cum_tiles_hit, tiles_x, tiles_y, 0, tiles_y, gaussian_ids_sorted, tile_bins,
                     workspace, workspace_bytes, stream, "igs_sort_intersects");
}

int igs_band_tiles_hit(int num_points, const float *xys, const int32_t *radii, int tiles_x, int tiles_y, int row_begin, int row_end,
                       int32_t *num_tiles_hit, void *stream) {
    IGS_REQUIRE(num_points >= 0 && tiles_x >= 0 && tiles_y >= 0, "igs_band_tiles_hit: negative size");
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "igs_band_tiles_hit: tile rows [%d, %d) outside [0, %d)",
                row_begin, row_end, tiles_y);
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(xys && radii && num_tiles_hit, "igs_band_tiles_hit: null pointer");
    IGS_REQUIRE(igs::aligned(xys, 8), "igs_band_tiles_hit: xys must be 8-byte aligned");
    igs::launch(band_hits_kernel, igs::ceil_div(num_points, 256), 256, 0, igs::as_stream(stream), num_points,
                reinterpret_cast<const float2 *>(xys), radii, (unsigned)tiles_x, (unsigned)tiles_y, (unsigned)row_begin, (unsigned)row_end,
                num_tiles_hit);
    return igs::check_launch("igs_band_tiles_hit");
}

int igs_sort_intersects_band(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit, int tiles_x,
                             int tiles_y, int row_begin, int row_end, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *workspace,
                             size_t workspace_bytes, void *stream) {
    return sort_band(num_points, capacity, xys, radii, cum_tiles_hit, tiles_x, tiles_y, row_begin, row_end, gaussian_ids_sorted, tile_bins,
                     workspace, workspace_bytes, stream, "igs_sort_intersects_band");
}

}  // extern "C"

namespace igs {

int cumsum_from_block_sums(int n, const int32_t *tiles_hit, const unsigned *block_sums, int32_t *cum, int32_t *total, cudaStream_t s) {
    static_assert(kCumBlock % 256 == 0, "block sums of 256 elements");
    if (n == 0) {
        if (total && cudaMemsetAsync(total, 0, sizeof(int), s) != cudaSuccess) return check_launch("prefix sum (training step)");
        return IGS_OK;
    }
    launch(cumsum_scan_kernel, ceil_div(n, kCumBlock), kCumThreads, 0, s, n, tiles_hit, block_sums, kCumBlock / 256, cum, total);
    return check_launch("prefix sum (training step)");
}

int sort_band_counters_zeroed(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit,
                              int tiles_x, int tiles_y, int row_begin, int row_end, int32_t *gaussian_ids_sorted, int32_t *tile_bins,
                              void *workspace, size_t workspace_bytes, cudaStream_t s) {
    return sort_band(num_points, capacity, xys, radii, cum_tiles_hit, tiles_x, tiles_y, row_begin, row_end, gaussian_ids_sorted, tile_bins,
                     workspace, workspace_bytes, s, "binning (training step)", true);
}

int *tile_counters(void *sort_workspace) { return static_cast<int *>(sort_workspace); }

}  // namespace igs

// ---- tile binning without device allocation -------------------------------------------------------------------------------------------
//
// For callers that cannot call cudaMalloc and have no workspace to lend: a plugin inside a host application that owns all device memory,
// or code running where an allocation would synchronize the device and stall its other streams. The scratch lives in a fixed array of
// this library instead, sized for IGS_NOALLOC_MAX_CAPACITY intersections over IGS_NOALLOC_MAX_TILES tiles (about 16 MiB). Every CUDA
// context that runs the library (the device's primary context, or a host application's own) holds one copy until the context or the
// process ends. All calls in a context share it: calls that overlap on the GPU (on different streams) race; what must start at zero
// (the per-tile counters) is cleared by every call. The first call in a context looks up the copy's address; make it before any stream
// capture in that context.

#include <cuda.h>

#include <mutex>
#include <utility>
#include <vector>

namespace {

constexpr size_t kNoAllocScratchBytes =
    ((sizeof(int) * (size_t)IGS_NOALLOC_MAX_TILES + 255) & ~(size_t)255) + 256 + ((sizeof(int2) * (size_t)IGS_NOALLOC_MAX_CAPACITY + 255) & ~(size_t)255) +
    2 * ((sizeof(int) * (size_t)IGS_NOALLOC_MAX_CAPACITY + 255) & ~(size_t)255);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// A __device__ array has one address per CUDA context, not per device: a host application may run this library under contexts of its
// own (cuCtxCreate / cuCtxSetCurrent) beside the device's primary one, and a context destroyed and created again (cudaDeviceReset, for
// one) gets new memory. So the address is cached per context, keyed by the context's ID (cuCtxGetId: unique for the life of the process,
// never reused, unlike the CUcontext handle). The two driver functions are reached through the runtime (cudaGetDriverEntryPoint), so
// the library does not link libcuda itself.
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

std::mutex g_noalloc_mutex;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
std::vector<std::pair<unsigned long long, void *>> g_noalloc_address;  // (context ID, the array's address in that context)

int noalloc_driver_entry_points() {
    if (g_ctx_get_current != nullptr && g_ctx_get_id != nullptr) return IGS_OK;
    void *get_current = nullptr, *get_id = nullptr;
    cudaDriverEntryPointQueryResult found_current = cudaDriverEntryPointSymbolNotFound, found_id = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &get_current, cudaEnableDefault, &found_current) != cudaSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &get_id, cudaEnableDefault, &found_id) != cudaSuccess ||
        found_current != cudaDriverEntryPointSuccess || found_id != cudaDriverEntryPointSuccess || !get_current || !get_id) {
        cudaGetLastError();
        return igs::set_error(IGS_ERR_UNSUPPORTED, "igs_sort_intersects_noalloc: the driver lacks cuCtxGetCurrent / cuCtxGetId");
    }
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(get_current);
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(get_id);
    return IGS_OK;
}

// The scratch array's device address in the calling thread's current context. In host code g_noalloc_scratch names a host-side
// stand-in, so the address is looked up (cudaGetSymbolAddress, with that context current) the first time a context calls, and cached.
// With no context current yet the runtime's lookup makes the current device's primary context current, as any runtime call would.
int noalloc_scratch(void **address) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    int status = noalloc_driver_entry_points();
    if (status != IGS_OK) return status;
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS)
        return igs::set_error(IGS_ERR_CUDA, "igs_sort_intersects_noalloc: cuCtxGetCurrent failed");
    void *p = nullptr;
    if (ctx == nullptr) {
        // no context yet on this thread: the runtime's lookup establishes the primary context, which is then current
        const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess)
            return igs::set_error(IGS_ERR_CUDA, "igs_sort_intersects_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
        if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
            return igs::set_error(IGS_ERR_CUDA, "igs_sort_intersects_noalloc: no current CUDA context");
    }
    unsigned long long id = 0;
    if (g_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return igs::set_error(IGS_ERR_CUDA, "igs_sort_intersects_noalloc: cuCtxGetId failed");
    for (const auto &entry : g_noalloc_address)
        if (entry.first == id) {
            *address = entry.second;
            return IGS_OK;
        }
    if (p == nullptr) {
        const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess)
            return igs::set_error(IGS_ERR_CUDA, "igs_sort_intersects_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
    }
    g_noalloc_address.emplace_back(id, p);
    *address = p;
    return IGS_OK;
}

}  // namespace

extern "C" int igs_sort_intersects_noalloc(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit,
                                           int tiles_x, int tiles_y, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *stream) {
    IGS_REQUIRE(capacity <= IGS_NOALLOC_MAX_CAPACITY,
                "igs_sort_intersects_noalloc: capacity %d exceeds the library's fixed scratch (at most %d intersections; use "
                "igs_sort_intersects with a workspace)", capacity, IGS_NOALLOC_MAX_CAPACITY);
    IGS_REQUIRE(tiles_x >= 0 && tiles_y >= 0 && (int64_t)tiles_x * tiles_y <= IGS_NOALLOC_MAX_TILES,
                "igs_sort_intersects_noalloc: %d x %d tiles exceed the library's fixed scratch (at most %d tiles; use igs_sort_intersects "
                "with a workspace)", tiles_x, tiles_y, IGS_NOALLOC_MAX_TILES);
    void *scratch = nullptr;
    const int status = noalloc_scratch(&scratch);
    if (status != IGS_OK) return status;
    return igs_sort_intersects(num_points, capacity, xys, radii, cum_tiles_hit, tiles_x, tiles_y, gaussian_ids_sorted, tile_bins, scratch,
                               kNoAllocScratchBytes, stream);
}
