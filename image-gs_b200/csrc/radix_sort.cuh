// A stable least-significant-digit radix sort of (64-bit key, int value) pairs on the GPU, 8 bits a pass and only as many passes as the
// keys are wide: per block of kTileKeys keys a digit histogram (count_kernel), one scan of all (digit, block) counts (scan_kernel), and a
// stable scatter (scatter_kernel: within a block, keys are ranked in order with per-warp __match_any_sync groups and a scan over the
// warps). Used by the bitstream order (order.cu) and the rate model's in-neighbour lists (rate_model.cu). Every definition is in an
// unnamed namespace, so each file including it has its own copy.
#pragma once

#include "igs_common.cuh"

namespace {
namespace radix {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 8;                       // keys per thread and pass
constexpr int kTileKeys = kThreads * kItems;    // keys per block
constexpr int kBins = 256;                      // 8-bit digits
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kThreads) count_kernel(const int n, const unsigned long long *__restrict__ keys, const int shift,
                                                         int *__restrict__ counts) {
    __shared__ int hist[kBins];
    hist[threadIdx.x] = 0;  // kThreads == kBins
    __syncthreads();
    const int base = blockIdx.x * kTileKeys;
    for (int e = base + threadIdx.x; e < min(n, base + kTileKeys); e += kThreads) atomicAdd(&hist[(keys[e] >> shift) & (kBins - 1)], 1);
    __syncthreads();
    counts[(size_t)threadIdx.x * gridDim.x + blockIdx.x] = hist[threadIdx.x];  // digit-major
}

// exclusive scan of counts[0, total) in place, one CTA in chunks of kScanThreads
__global__ void __launch_bounds__(kScanThreads) scan_kernel(const int total, int *__restrict__ counts) {
    __shared__ int warp_sums[kScanThreads / 32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < total; base += kScanThreads) {
        const int i = base + threadIdx.x;
        const int v = i < total ? counts[i] : 0;
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = warp_sums[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += t;
            }
            warp_sums[lane] = w;
        }
        __syncthreads();
        const int before = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
        if (i < total) counts[i] = before + incl - v;
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[kScanThreads / 32 - 1];
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads) scatter_kernel(const int n, const unsigned long long *__restrict__ keys_in,
                                                           const int *__restrict__ idx_in, const int shift, const int *__restrict__ offsets,
                                                           unsigned long long *__restrict__ keys_out, int *__restrict__ idx_out) {
    __shared__ int running[kBins];          // the next place of each digit for this block
    __shared__ int wcount[kWarps][kBins];   // per warp and digit: the count, then the warp's first place
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    running[threadIdx.x] = offsets[(size_t)threadIdx.x * gridDim.x + blockIdx.x];
    const int base = blockIdx.x * kTileKeys;
    for (int s = 0; s < kItems; ++s) {
        const int e = base + s * kThreads + threadIdx.x;
        const bool valid = e < n;
        const unsigned long long key = valid ? keys_in[e] : 0ull;
        const int d = valid ? (int)((key >> shift) & (kBins - 1)) : kBins;  // kBins: no key
#pragma unroll
        for (int w = 0; w < kWarps; ++w) wcount[w][threadIdx.x] = 0;
        __syncthreads();
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (valid && rank == 0) wcount[warp][d] = __popc(peers);
        __syncthreads();
        {
            int acc = running[threadIdx.x];
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const int c = wcount[w][threadIdx.x];
                wcount[w][threadIdx.x] = acc;
                acc += c;
            }
            running[threadIdx.x] = acc;
        }
        __syncthreads();
        if (valid) {
            const int place = wcount[warp][d] + rank;
            keys_out[place] = key;
            idx_out[place] = idx_in[e];
        }
        __syncthreads();
    }
}

// Workspace of a sort of n pairs besides the two key and two value buffers: the (digit, block) counts
inline size_t counts_bytes(int n) { return sizeof(int) * kBins * (size_t)igs::ceil_div(n > 0 ? n : 1, kTileKeys); }

// Sorts keys[0] / values[0] (n pairs) by the low key_bits bits of the keys, stably, ping-ponging through keys[1] / values[1]; returns the
// index (0 or 1) of the buffers holding the result
inline int sort_pairs(const int n, const int key_bits, unsigned long long *keys[2], int *values[2], int *counts, cudaStream_t s) {
    const int tile_blocks = igs::ceil_div(n, kTileKeys);
    int cur = 0;
    for (int shift = 0; shift < key_bits; shift += 8) {
        count_kernel<<<tile_blocks, kThreads, 0, s>>>(n, keys[cur], shift, counts);
        scan_kernel<<<1, kScanThreads, 0, s>>>(kBins * tile_blocks, counts);
        scatter_kernel<<<tile_blocks, kThreads, 0, s>>>(n, keys[cur], values[cur], shift, counts, keys[1 - cur], values[1 - cur]);
        cur = 1 - cur;
    }
    return cur;
}

inline int bit_length(unsigned long long v) {
    int b = 0;
    while (v) ++b, v >>= 1;
    return b;
}

}  // namespace radix
}  // namespace
