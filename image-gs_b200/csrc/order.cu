// The bitstream order of the Gaussians (compress/__init__.py:43-58, bitstream_order, with the Morton interleave of compress/common.py:87-97):
// along the Morton curve of the positions coarsened by refine_bits (positions >> refine_bits, minus their minimum), ties by the Morton code
// of the full positions (minus their minimum), then by index. The reference sorts on the host with numpy; here:
//   1. minmax_kernel: the positions' range (read back once: it sets the key width, and positions spanning 2^32 levels or more are
//      rejected as the reference rejects them);
//   2. keys_kernel: one 64-bit key per Gaussian, the coarse Morton code above the fine one (their order is the lexicographic order of
//      the pair), with its index;
//   3. a stable least-significant-digit radix sort of the keys over the key's width only (radix_sort.cuh).
// A pair of codes wider than 64 bits in all (coordinates spanning more than 2^16 coarse and fine levels together) is reported as
// IGS_ERR_UNSUPPORTED for the caller's host sort.
#include <climits>

#include "igs_common.cuh"
#include "radix_sort.cuh"

namespace {

using radix::kThreads;
using radix::kWarps;

struct Range {
    long long min_x, min_y, max_x, max_y;
};

__device__ __forceinline__ unsigned long long part1by1(unsigned long long x) {
    // the lower 32 bits of x spread to the even bit positions
    x &= 0xFFFFFFFFull;
    x = (x | (x << 16)) & 0x0000FFFF0000FFFFull;
    x = (x | (x << 8)) & 0x00FF00FF00FF00FFull;
    x = (x | (x << 4)) & 0x0F0F0F0F0F0F0F0Full;
    x = (x | (x << 2)) & 0x3333333333333333ull;
    x = (x | (x << 1)) & 0x5555555555555555ull;
    return x;
}

__device__ __forceinline__ unsigned long long morton(long long x, long long y) {
    return part1by1((unsigned long long)x) | (part1by1((unsigned long long)y) << 1);
}

__global__ void init_range_kernel(Range *r) {
    r->min_x = r->min_y = LLONG_MAX;
    r->max_x = r->max_y = LLONG_MIN;
}

__global__ void __launch_bounds__(kThreads) minmax_kernel(const int n, const long long *__restrict__ pos, Range *__restrict__ r) {
    __shared__ long long s[4][kWarps];
    long long v[4] = {LLONG_MAX, LLONG_MAX, LLONG_MIN, LLONG_MIN};
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
        const long long x = pos[2 * (size_t)i], y = pos[2 * (size_t)i + 1];
        v[0] = min(v[0], x), v[1] = min(v[1], y), v[2] = max(v[2], x), v[3] = max(v[3], y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v[0] = min(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
        v[1] = min(v[1], __shfl_xor_sync(0xffffffffu, v[1], o));
        v[2] = max(v[2], __shfl_xor_sync(0xffffffffu, v[2], o));
        v[3] = max(v[3], __shfl_xor_sync(0xffffffffu, v[3], o));
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0)
        for (int k = 0; k < 4; ++k) s[k][warp] = v[k];
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kWarps; ++w) {
            v[0] = min(v[0], s[0][w]), v[1] = min(v[1], s[1][w]);
            v[2] = max(v[2], s[2][w]), v[3] = max(v[3], s[3][w]);
        }
        atomicMin(&r->min_x, v[0]), atomicMin(&r->min_y, v[1]);
        atomicMax(&r->max_x, v[2]), atomicMax(&r->max_y, v[3]);
    }
}

__global__ void __launch_bounds__(kThreads) keys_kernel(const int n, const long long *__restrict__ pos, const int refine_bits,
                                                        const long long coarse_x0, const long long coarse_y0, const long long fine_x0,
                                                        const long long fine_y0, const int fine_bits, unsigned long long *__restrict__ keys,
                                                        int *__restrict__ idx) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;
    const long long x = pos[2 * (size_t)i], y = pos[2 * (size_t)i + 1];
    const unsigned long long fine = morton(x - fine_x0, y - fine_y0);
    keys[i] = refine_bits == 0 ? fine : (morton((x >> refine_bits) - coarse_x0, (y >> refine_bits) - coarse_y0) << fine_bits) | fine;
    idx[i] = i;
}

__global__ void __launch_bounds__(kThreads) widen_kernel(const int n, const int *__restrict__ idx, long long *__restrict__ order) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i < n) order[i] = idx[i];
}

struct Layout {
    size_t range, keys0, keys1, idx0, idx1, counts, total;
};

Layout layout(int n) {
    const size_t num = n > 0 ? (size_t)n : 1;
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    Layout l;
    size_t off = 0;
    l.range = off, off += up(sizeof(Range));
    l.keys0 = off, off += up(sizeof(unsigned long long) * num);
    l.keys1 = off, off += up(sizeof(unsigned long long) * num);
    l.idx0 = off, off += up(sizeof(int) * num);
    l.idx1 = off, off += up(sizeof(int) * num);
    l.counts = off, off += up(radix::counts_bytes((int)num));
    l.total = off;
    return l;
}

}  // namespace

extern "C" {

size_t igs_bitstream_order_workspace(int num_points) { return layout(num_points).total; }

int igs_bitstream_order(int num_points, const int64_t *positions, int refine_bits, int64_t *order, void *workspace, size_t workspace_bytes,
                        void *stream) {
    const char *who = "igs_bitstream_order";
    IGS_REQUIRE(num_points >= 0, "%s: negative size", who);
    IGS_REQUIRE(refine_bits >= 0 && refine_bits < 32, "%s: refine_bits %d outside [0, 32)", who, refine_bits);
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(positions && order && workspace, "%s: null pointer", who);
    IGS_REQUIRE(igs::aligned(positions, 16), "%s: positions must be 16-byte aligned [P, 2] int64", who);
    const Layout l = layout(num_points);
    IGS_REQUIRE(workspace_bytes >= l.total, "%s: workspace too small (%zu bytes, need %zu)", who, workspace_bytes, l.total);
    IGS_REQUIRE(igs::aligned(workspace, 256), "%s: workspace must be 256-byte aligned", who);
    cudaStream_t s = igs::as_stream(stream);
    char *ws = static_cast<char *>(workspace);
    Range *range = reinterpret_cast<Range *>(ws + l.range);
    unsigned long long *keys[2] = {reinterpret_cast<unsigned long long *>(ws + l.keys0), reinterpret_cast<unsigned long long *>(ws + l.keys1)};
    int *idx[2] = {reinterpret_cast<int *>(ws + l.idx0), reinterpret_cast<int *>(ws + l.idx1)};
    int *counts = reinterpret_cast<int *>(ws + l.counts);
    const long long *pos = reinterpret_cast<const long long *>(positions);
    const int elem_blocks = igs::ceil_div(num_points, kThreads);

    // 1. the range, read back once
    init_range_kernel<<<1, 1, 0, s>>>(range);
    minmax_kernel<<<std::min(elem_blocks, 148 * 4), kThreads, 0, s>>>(num_points, pos, range);
    Range r;
    if (cudaMemcpyAsync(&r, range, sizeof(Range), cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return igs::check_launch(who);
    const long long cx0 = r.min_x >> refine_bits, cy0 = r.min_y >> refine_bits;
    const unsigned long long coarse_span = (unsigned long long)std::max((r.max_x >> refine_bits) - cx0, (r.max_y >> refine_bits) - cy0);
    IGS_REQUIRE(coarse_span < (1ull << 32), "%s: the positions must have at most 2^32 quantization levels per coordinate", who);
    const unsigned long long fine_span = (unsigned long long)std::max(r.max_x - r.min_x, r.max_y - r.min_y);
    if (refine_bits > 0 && fine_span >= (1ull << 32)) return igs::set_error(IGS_ERR_UNSUPPORTED, "%s: fine positions over 2^32 levels", who);
    const int fine_bits = 2 * radix::bit_length(fine_span);
    const int key_bits = refine_bits == 0 ? fine_bits : 2 * radix::bit_length(coarse_span) + fine_bits;
    if (key_bits > 64) return igs::set_error(IGS_ERR_UNSUPPORTED, "%s: a %d-bit sort key (sort on the host)", who, key_bits);

    // 2. keys and indices
    keys_kernel<<<elem_blocks, kThreads, 0, s>>>(num_points, pos, refine_bits, cx0, cy0, r.min_x, r.min_y, fine_bits, keys[0], idx[0]);
    // 3. stable radix passes over the key's width
    const int cur = radix::sort_pairs(num_points, key_bits, keys, idx, counts, s);
    widen_kernel<<<elem_blocks, kThreads, 0, s>>>(num_points, idx[cur], reinterpret_cast<long long *>(order));
    return igs::check_launch(who);
}

}  // extern "C"
