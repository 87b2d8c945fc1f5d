// Top-K normalized rasterization of 2D Gaussians, forward and backward, for 16x16 tiles.
//
// Forward (the semantics of nd_rasterize_forward_topk_norm, gsplat/gsplat/cuda/csrc/forward.cu:223-375): every pixel walks its tile's
// Gaussian list in order and keeps the 10 largest alpha = exp(-sigma), sigma = (a dx^2 + c dy^2) / 2 + b dx dy, skipping sigma < 0, NaN or
// Inf. A Gaussian enters if its alpha exceeds the cached minimum (-1 while slots are free): into the next free slot, or else into the first
// slot holding the strict minimum, after which the minimum is rescanned. The pixel's value is sum_k f_k alpha_k / (sum_k alpha_k + 1e-4),
// accumulated over the slots in slot order. Slot order and contents are part of the output (pixel_topk), so the insertion rule is kept
// exactly.
//
// B200 layout: one CTA per tile (grid = tiles, so the hardware balances uneven list lengths over the 148 SMs); pixels are numbered so
// that 32 consecutive ones form a compact 8x4 patch; the forward's 128 threads take two pixels each (patches t and t + 128), the
// backward's 256 threads one; the tile's list is staged in shared memory in chunks of 256 entries (one 16-byte and one 4-byte broadcast
// load per Gaussian, shared by a thread's pixels). The forward can also take the L1 loss of its pixels and write the loss's gradient with
// respect to the image. The training step runs forward, L1 loss and backward of a tile in one kernel (raster_step_kernel, 256 threads,
// one pixel each), keeping the top-K lists and the image gradient on chip. Two output forms of the top-K lists of the separate forward:
//   * pixel_topk [H, W, 10] int32 Gaussian IDs (the reference's operator output), written through shared memory as coalesced 8-byte rows;
//   * tile lists (autograd path): per tile, slot-major [10][256] uint16 positions in the tile's Gaussian list, 20 bytes per pixel instead
//     of 40, written as coalesced 64-byte warp rows, and read back by the backward pass, which stages the same list in shared memory.
// Compiled with --use_fast_math like the reference (__expf, approximate division), so alpha values and hence the lists match bit for bit.
//
// Backward (the math of nd_rasterize_backward_topk_norm_kernel, backward.cu:187-308): with D = 1e-4 + sum_k d_k and s_k = f_k . v_out,
// v_sigma_k = -d_k (s_k / D - sum_j d_j s_j / D^2) and the colour weight d_k / D; per Gaussian v_conic += (v_sigma dx^2 / 2, v_sigma dx dy,
// v_sigma dy^2 / 2), v_xy += v_sigma (a dx + b dy, b dx + c dy), v_color += (d_k / D) v_out. Two kernels and the fused one:
//   * raster_bwd_pairs_kernel (autograd path, from the tile lists): the tile's (pixel, slot) pairs grouped by Gaussian in shared memory,
//     one warp per Gaussian summing its pairs, then one global atomic per (tile, Gaussian, value); see the comment above it (the fused
//     raster_step_kernel ends with the same steps);
//   * raster_bwd_ids_kernel (the [H, W, 10] operator): each warp visits the union of its 32 pixels' top-K Gaussian IDs in increasing
//     order (a warp-wide minimum per step), sums the 5 + C values of each over the warp with a recursive-halving reduce-scatter, and
//     adds them with one global atomic per value.
#include <algorithm>
#include <cstddef>

#include "igs_common.cuh"
#include "igs_internal.cuh"

namespace {

using igs::kMaxChannels;
using igs::kNoSlot;
using igs::kTile;
using igs::kTilePixels;
using igs::kTopK;

constexpr int kThreads = kTilePixels;  // pixels of a tile (and threads of the backward's CTA)
constexpr int kChunk = 256;            // list entries staged per round in the forward pass
constexpr int kPairStage = 256;        // longest tile list of the pairs-grouped backward pass
// the fused step kernel keeps the selection's last staged chunk for its backward part: both passes stage the same chunks
static_assert(kChunk == kPairStage, "the forward and backward passes must stage the same chunks of a tile's list");
constexpr int kPairs = kThreads * kTopK;
struct PixelCoord {
    int i, j;  // row, column in the image
    int tid;   // thread / pixel index within the tile
};

// Warp w covers the 8x4 patch (w % 2, w / 2) of the tile; lane l its pixel (l % 8, l / 8). lid is the pixel's index in this layout
// (0..255). Tiles are numbered within a band of tile rows starting at row_begin (0 for the whole image); the coordinates are the image's.
__device__ __forceinline__ PixelCoord tile_pixel_of(int tile, int tiles_x, int row_begin, int lid) {
    const int lane = lid & 31, warp = lid >> 5;
    const int lx = (warp & 1) * 8 + (lane & 7), ly = (warp >> 1) * 4 + (lane >> 3);
    return {(row_begin + tile / tiles_x) * kTile + ly, (tile % tiles_x) * kTile + lx, lid};
}

// one pixel per thread
__device__ __forceinline__ PixelCoord tile_pixel(int tile, int tiles_x, int row_begin) {
    return tile_pixel_of(tile, tiles_x, row_begin, threadIdx.x);
}


// The reference skips an entry whose sigma is negative, NaN or infinite (forward.cu:301)
__device__ __forceinline__ bool sigma_valid(const float sigma) { return !(sigma < 0.f || isnan(sigma) || isinf(sigma)); }

// sigma of one pixel from a Gaussian's centre and halved conic (g4 = x, y, a / 2, b; hc = c / 2): the same roundings as
// igs::gaussian_sigma, since halving is exact (0.5 fma(a dx, dx, (c dy) dy) = fma(ha dx, dx, (hc dy) dy))
__device__ __forceinline__ float halved_sigma(const float4 g4, const float hc, const float px, const float py) {
    const float dx = __fsub_rn(g4.x, px), dy = __fsub_rn(g4.y, py);
    return __fmaf_rn(__fmul_rn(g4.w, dx), dy, __fmaf_rn(__fmul_rn(g4.z, dx), dx, __fmul_rn(__fmul_rn(hc, dy), dy)));
}

// The selection stages a chunk of the tile's list in pairs of entries, so that one packed (f32x2) instruction serves two entries: pair i
// (entries 2i, 2i + 1) is geo[2i] = (x0, x1, y0, y1) and geo[2i + 1] = (a0 / 2, a1 / 2, b0, b1); cc[e] = c / 2 of entry e. The packed
// instructions round each component like their scalar forms, so the sigma values are those of halved_sigma bit for bit.
__device__ __forceinline__ void stage_paired(float4 *geo, float *cc, const int e, const float2 xy, const float a, const float b,
                                             const float c) {
    float *g = reinterpret_cast<float *>(geo) + 8 * (e >> 1) + (e & 1);
    g[0] = xy.x;
    g[2] = xy.y;
    g[4] = 0.5f * a;
    g[6] = b;
    cc[e] = 0.5f * c;
}

// one entry of the paired layout: (x, y, a / 2, b)
__device__ __forceinline__ float4 paired_geo(const float4 *geo, const int e) {
    const float *g = reinterpret_cast<const float *>(geo) + 8 * (e >> 1) + (e & 1);
    return make_float4(g[0], g[2], g[4], g[6]);
}

// sigma of two consecutive entries (a pair of the paired layout: p = (x0, x1, y0, y1), h = (a0 / 2, a1 / 2, b0, b1), hc = (c0 / 2,
// c1 / 2)) at PPT pixels of one column; npx = (-px, -px) and npy[q] = (-py, -py) (x - p is x + (-p) exactly)
template <int PPT>
__device__ __forceinline__ void pair_sigma(const float4 p, const float4 h, const float2 hc, const float2 npx, const float2 (&npy)[PPT],
                                           float2 (&sigma)[PPT]) {
    const float2 dx = __fadd2_rn(make_float2(p.x, p.y), npx);
    const float2 adx = __fmul2_rn(make_float2(h.x, h.y), dx), bdx = __fmul2_rn(make_float2(h.z, h.w), dx);
#pragma unroll
    for (int q = 0; q < PPT; ++q) {
        const float2 dy = __fadd2_rn(make_float2(p.z, p.w), npy[q]);
        sigma[q] = __ffma2_rn(bdx, dy, __ffma2_rn(adx, dx, __fmul2_rn(__fmul2_rn(hc, dy), dy)));
    }
}

// u += d f over the channels, in pairs of channels with packed instructions (each component rounded as fmaf)
template <int kMaxC>
__device__ __forceinline__ void add_weighted(const float d, const float (&f)[kMaxC], float (&u)[kMaxC]) {
#pragma unroll
    for (int c = 0; c + 1 < kMaxC; c += 2) {
        const float2 r = __ffma2_rn(make_float2(d, d), make_float2(f[c], f[c + 1]), make_float2(u[c], u[c + 1]));
        u[c] = r.x, u[c + 1] = r.y;
    }
    if (kMaxC & 1) u[kMaxC - 1] = fmaf(d, f[kMaxC - 1], u[kMaxC - 1]);
}

// The top-K selection of PPT pixels per thread over their tile's list (range into ids_sorted), in list order, with the slot rule of the
// reference: free slots take valid entries in order, then an entry whose alpha exceeds the minimum replaces the first slot holding it.
// The first ten entries fill the slots with fixed indices when all of them are valid for a pixel (what the rule does while slots are
// free); only a pixel that cannot take that path starts from empty slots. The list is staged through s_geo / s_cc (paired layout, see
// stage_paired) in chunks of kChunk entries by the CTA's kThreads / PPT threads, with CTA barriers: every thread must call it; a chunk of
// odd length gets a NaN entry after its last, which no pixel takes. The entries are evaluated two at a time with packed instructions,
// then tested in list order. The slots live in shared memory, alpha in
// s_val and the list position in s_pos (both [k * kThreads + lid], position -1 for empty), so an insertion is two dynamic stores instead
// of a select over ten registers; each pixel keeps the minimum of each half of its slots (0-4, 5-9) and the first slot holding it in
// registers, so that an insertion rescans only the half it wrote (the first slot of the strict minimum over all ten is the second
// half's only if that half's minimum is strictly smaller). The staged conic is halved (exactly), which drops a multiplication from
// sigma, and the PPT pixels of a thread share a column, so dx and its products are shared too. On return val[q][k] holds the slots'
// alpha. Pixels outside the image (inside[q] false) take no entries.
template <int PPT>
__device__ __forceinline__ void select_topk(const int2 range, const int *__restrict__ ids_sorted, const float2 *__restrict__ xys,
                                            const float *__restrict__ conics, const PixelCoord (&pc)[PPT], const bool (&inside)[PPT],
                                            float4 *s_geo, float *s_cc, int *s_pos, float *s_val, float (&val)[PPT][kTopK]) {
    constexpr int kStagers = kThreads / PPT;
    constexpr int kHalf = kTopK / 2;
    static_assert(kTopK % 2 == 0 && kChunk % 2 == 0, "entries are evaluated in pairs");
    const int tid = threadIdx.x;
    const int len = range.y - range.x;
    const float px = (float)pc[0].j;  // the pixels share a column
    const float2 npx = make_float2(-px, -px);
    float2 npy[PPT];
    float min_val[PPT];
    int filled[PPT];
    float gv[PPT][2];  // per half of the slots (0-4, 5-9): its minimum and the first slot holding it
    int gs[PPT][2];
    auto clear_slots = [&](const int q) {
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            s_pos[k * kThreads + pc[q].tid] = -1;
            s_val[k * kThreads + pc[q].tid] = 0.f;
        }
    };
#pragma unroll
    for (int q = 0; q < PPT; ++q) {
        npy[q] = make_float2(-(float)pc[q].i, -(float)pc[q].i);
        filled[q] = inside[q] ? 0 : kTopK;  // a pixel outside the image counts as full with an unbeatable minimum
        min_val[q] = inside[q] ? -1.f : INFINITY;
        if (len <= 0) clear_slots(q);  // no chunk below: the slots stay empty
    }
    // minimum of one half of a pixel's slots (the first slot on ties)
    auto scan_half = [&](const int q, const int h) {
        const float *v = s_val + h * kHalf * kThreads + pc[q].tid;
        float m = v[0];
        int ms = 0;
#pragma unroll
        for (int k = 1; k < kHalf; ++k) {
            const float x = v[k * kThreads];
            if (x < m) m = x, ms = k;
        }
        return make_float2(m, __int_as_float(ms + h * kHalf));
    };
    auto rescan = [&](const int q) {
        const float2 h0 = scan_half(q, 0), h1 = scan_half(q, 1);
        gv[q][0] = h0.x, gs[q][0] = __float_as_int(h0.y);
        gv[q][1] = h1.x, gs[q][1] = __float_as_int(h1.y);
        min_val[q] = fminf(gv[q][0], gv[q][1]);
    };
    // replace the first slot holding the minimum (the second half's only if strictly smaller), then rescan that half
    auto insert = [&](const int q, const float alpha, const int position) {
        const int h = gv[q][1] < gv[q][0] ? 1 : 0;
        const int slot = h ? gs[q][1] : gs[q][0];
        s_pos[slot * kThreads + pc[q].tid] = position;
        s_val[slot * kThreads + pc[q].tid] = alpha;
        const float2 m = scan_half(q, h);
        if (h) gv[q][1] = m.x, gs[q][1] = __float_as_int(m.y);
        else gv[q][0] = m.x, gs[q][0] = __float_as_int(m.y);
        min_val[q] = fminf(gv[q][0], gv[q][1]);
    };
    auto all_full = [&]() {
        bool full = true;
#pragma unroll
        for (int q = 0; q < PPT; ++q) full = full && filled[q] == kTopK;
        return full;
    };

    for (int base = 0; base < len; base += kChunk) {
        const int count = min(kChunk, len - base);
        __syncthreads();
        for (int i = tid; i < count; i += kStagers) {
            const int g = __ldg(&ids_sorted[range.x + base + i]);
            stage_paired(s_geo, s_cc, i, __ldg(&xys[g]), __ldg(&conics[3 * g]), __ldg(&conics[3 * g + 1]), __ldg(&conics[3 * g + 2]));
        }
        if ((count & 1) && tid == 0) stage_paired(s_geo, s_cc, count, make_float2(NAN, NAN), NAN, NAN, NAN);  // odd length: a NaN entry
        __syncthreads();
        int start[PPT];  // first entry of the chunk each pixel still has to consider (0 or kTopK: even)
#pragma unroll
        for (int q = 0; q < PPT; ++q) start[q] = 0;
        if (base == 0) {
            // fast fill, per pixel: all of the first ten entries valid -> slots 0..9 in order, with the half minima kept as the slots are
            // written; a pixel with an invalid entry among them (or a shorter list, or outside the image) clears them and starts from
            // empty slots below
            bool fast[PPT];
#pragma unroll
            for (int q = 0; q < PPT; ++q) fast[q] = count >= kTopK && inside[q];
            if (count >= kTopK) {
#pragma unroll
                for (int k = 0; k < kTopK; k += 2) {
                    float2 s2[PPT];
                    pair_sigma<PPT>(s_geo[k], s_geo[k + 1], *reinterpret_cast<const float2 *>(&s_cc[k]), npx, npy, s2);
#pragma unroll
                    for (int q = 0; q < PPT; ++q) {
#pragma unroll
                        for (int o = 0; o < 2; ++o) {
                            const int kk = k + o;
                            const float sk = o ? s2[q].y : s2[q].x;
                            fast[q] = fast[q] && sigma_valid(sk);
                            const float a = __expf(-sk);
                            s_val[kk * kThreads + pc[q].tid] = a;
                            s_pos[kk * kThreads + pc[q].tid] = kk;
                            const int h = kk / kHalf;
                            if (kk % kHalf == 0 || a < gv[q][h]) gv[q][h] = a, gs[q][h] = kk;
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < PPT; ++q) {
                if (!fast[q]) {
                    clear_slots(q);
                    if (!inside[q] && count >= kTopK) start[q] = kTopK;  // never inserts: keeps the pixels' starts equal below
                    continue;
                }
                min_val[q] = fminf(gv[q][0], gv[q][1]);
                filled[q] = kTopK;
                start[q] = kTopK;
            }
        }
        int e = start[0];
#pragma unroll
        for (int q = 1; q < PPT; ++q) e = min(e, start[q]);
        if (all_full()) {
            // the common case: every pixel full (all starts equal), only the replacement rule
            for (; e < count; e += 2) {
                float2 s2[PPT];
                pair_sigma<PPT>(s_geo[e], s_geo[e + 1], *reinterpret_cast<const float2 *>(&s_cc[e]), npx, npy, s2);
#pragma unroll
                for (int q = 0; q < PPT; ++q) {
                    // every slot holds an alpha >= 0 (the minimum of a pixel outside the image is infinite), so sigma >= 0 suffices: an
                    // infinite sigma gives alpha = 0, which replaces nothing, and NaN (also the padding entry) fails the test
                    const float a0 = __expf(-s2[q].x), a1 = __expf(-s2[q].y);
                    if (s2[q].x >= 0.f && a0 > min_val[q]) insert(q, a0, base + e);
                    if (s2[q].y >= 0.f && a1 > min_val[q]) insert(q, a1, base + e + 1);
                }
            }
        } else {
            for (; e < count; e += 2) {
                float2 s2[PPT];
                pair_sigma<PPT>(s_geo[e], s_geo[e + 1], *reinterpret_cast<const float2 *>(&s_cc[e]), npx, npy, s2);
#pragma unroll
                for (int q = 0; q < PPT; ++q) {
                    if (e < start[q]) continue;  // starts are even: both entries of the pair or neither
#pragma unroll
                    for (int o = 0; o < 2; ++o) {
                        const float sigma = o ? s2[q].y : s2[q].x;
                        if (!sigma_valid(sigma)) continue;  // also the padding entry
                        const float alpha = __expf(-sigma);
                        if (filled[q] < kTopK) {
                            s_val[filled[q] * kThreads + pc[q].tid] = alpha;
                            s_pos[filled[q] * kThreads + pc[q].tid] = base + e + o;
                            if (++filled[q] == kTopK) rescan(q);
                        } else if (alpha > min_val[q]) {
                            insert(q, alpha, base + e + o);
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int q = 0; q < PPT; ++q)
#pragma unroll
        for (int k = 0; k < kTopK; ++k) val[q][k] = s_val[k * kThreads + pc[q].tid];
}

// The L1 loss of the rendered pixels fused into the forward pass (the training loss of model.py:1224-1227, ratio * F.l1_loss(image,
// target), and its gradient sign(image - target) * ratio / numel): each CTA writes the gradient of its pixels and the sum of their
// |image - target| (in a fixed order) to partials[tile]; l1_finish_kernel, launched next, adds the partials in tile order, so the loss
// is deterministic. (Forming the loss in the last CTA to finish would make every CTA wait for a returning atomic before it exits: at
// 8,160 tiles that costs more than the second launch.) target == nullptr: no loss.
struct FusedL1 {
    const float *target;  // [C, rows, W] like the image (the band's rows for a band)
    float *v_output;      // gradient of the loss with respect to the image, same layout
    float grad_value;     // ratio / numel (numel of the whole image)
    float *partials;      // one per tile of the launch
};

__device__ __forceinline__ float l1_sign(float d) { return d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f); }

// Sum of one value per thread over the CTA (blockDim.x threads, a multiple of 32) in a fixed order; the result is valid in thread 0.
// scratch: blockDim.x / 32 floats.
__device__ __forceinline__ float cta_sum(float v, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // scratch may still be read by a previous use
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.f;
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += scratch[w];
    return total;
}

constexpr int kFinishThreads = 1024;

// loss = ratio * (sum of the partials in tile order) / numel, one CTA
__global__ void __launch_bounds__(kFinishThreads) l1_finish_kernel(const float *__restrict__ partials, const int count, const float ratio,
                                                                   const float numel, float *__restrict__ loss) {
    igs::wait_for_predecessor();
    __shared__ float scratch[kFinishThreads / 32];
    float sum = 0.f;
#pragma unroll 8
    for (int t = threadIdx.x; t < count; t += kFinishThreads) sum += __ldg(&partials[t]);
    const float all = cta_sum(sum, scratch);
    if (threadIdx.x == 0) *loss = ratio * (all / numel);
}

// Pixels per thread of the forward pass: two (a thread takes the pixels of lane ids t and t + 128 of the tile layout: the same column,
// eight rows apart), sharing the staged Gaussians' loads, dx and the loop, and 128 threads per tile.
constexpr int kFwdPixels = 2;
constexpr int kFwdThreads = kThreads / kFwdPixels;

template <int C>
__global__ void __launch_bounds__(kFwdThreads, 8)
    raster_fwd_kernel(const int tiles_x, const int img_h, const int img_w, const int row_begin, const int band_h, const int channels_rt,
        const int *__restrict__ ids_sorted, const int2 *__restrict__ tile_bins, const float2 *__restrict__ xys,
        const float *__restrict__ conics, const float *__restrict__ colors, float *__restrict__ out_img, int *__restrict__ pixel_topk,
        uint16_t *__restrict__ tile_topk, const FusedL1 l1) {
    igs::wait_for_predecessor();
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    __shared__ float4 s_geo[kChunk];         // x, y, conic a / 2, conic b; then the colours of a one-chunk list
    __shared__ __align__(16) float s_cc[kChunk];  // conic c / 2
    __shared__ int s_ids[kThreads * kTopK];  // the slots' list positions during the selection, then the IDs of [H, W, 10] lists

    const int tile = blockIdx.x;
    PixelCoord pc[kFwdPixels];
    bool inside[kFwdPixels];
#pragma unroll
    for (int q = 0; q < kFwdPixels; ++q) {
        pc[q] = tile_pixel_of(tile, tiles_x, row_begin, threadIdx.x + q * kFwdThreads);
        inside[q] = pc[q].i < img_h && pc[q].j < img_w;
    }
    const int2 range = tile_bins[tile];
    const int len = range.y - range.x;

    float val[kFwdPixels][kTopK];
    __shared__ float s_val[kThreads * kTopK];  // the slots' alpha values during the selection
    select_topk<kFwdPixels>(range, ids_sorted, xys, conics, pc, inside, s_geo, s_cc, s_ids, s_val, val);

    const int num_pixels = band_h * img_w;  // one channel plane of the (band of the) image
    const bool addressable = len < (int)kNoSlot;
    // a list of one chunk: its colours replace the staged geometry in shared memory, read by list position below
    constexpr bool kStageColors = C > 0 && C <= 4;
    const bool colors_staged = kStageColors && len <= kChunk;
    if (colors_staged) {
        __syncthreads();
        for (int e = threadIdx.x; e < len; e += kFwdThreads) {
            const float *f = colors + (size_t)__ldg(&ids_sorted[range.x + e]) * channels;
            s_geo[e] = make_float4(__ldg(&f[0]), C > 1 ? __ldg(&f[1]) : 0.f, C > 2 ? __ldg(&f[2]) : 0.f, C > 3 ? __ldg(&f[3]) : 0.f);
        }
        __syncthreads();
    }
    float acc = 0.f;  // the CTA's part of the L1 loss
#pragma unroll
    for (int q = 0; q < kFwdPixels; ++q) {
        int pos[kTopK], gid[kTopK];
#pragma unroll
        for (int k = 0; k < kTopK; ++k) pos[k] = s_ids[k * kThreads + pc[q].tid];
        // the normalized sum U / D: U = sum_k d_k f_k and D = 1e-4 + sum_k d_k accumulated in slot order, one reciprocal (within a few
        // float roundings of the reference's per-slot double-precision division; the training step's kernel computes the same)
        float denom = (float)igs::kNormEps;
        float pix[kMaxC];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) pix[c] = 0.f;
        if (colors_staged) {
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                if (pos[k] < 0) continue;
                const float d = val[q][k];
                denom += d;
                const float4 f4 = s_geo[pos[k]];
                const float fa[4] = {f4.x, f4.y, f4.z, f4.w};
                float f[kMaxC];
#pragma unroll
                for (int c = 0; c < kMaxC; ++c) f[c] = fa[c < 4 ? c : 0];
                add_weighted(d, f, pix);
            }
        } else {
#pragma unroll
            for (int k = 0; k < kTopK; ++k) gid[k] = pos[k] >= 0 ? __ldg(&ids_sorted[range.x + pos[k]]) : -1;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                if (gid[k] < 0) continue;
                const float d = val[q][k];
                denom += d;
                const float *f = colors + (size_t)gid[k] * channels;
#pragma unroll
                for (int c = 0; c < kMaxC; ++c)
                    if (c < channels) pix[c] = fmaf(d, __ldg(&f[c]), pix[c]);
            }
        }
        const float inv_denom = 1.f / denom;
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) pix[c] *= inv_denom;
        const int p = (pc[q].i - row_begin * kTile) * img_w + pc[q].j;
        if (inside[q]) {
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) {
                if (c >= channels) continue;
                out_img[(size_t)c * num_pixels + p] = pix[c];
                if (l1.target != nullptr) {
                    const float d = pix[c] - __ldcs(&l1.target[(size_t)c * num_pixels + p]);
                    acc += fabsf(d);
                    __stcs(&l1.v_output[(size_t)c * num_pixels + p], l1_sign(d) * l1.grad_value);
                }
            }
        }
        if (tile_topk != nullptr) {
            // a tile whose list holds 65535 entries or more is left empty: raster_bwd_pairs_kernel selects its lists again
            uint16_t *dst = tile_topk + (size_t)tile * kTopK * kThreads + pc[q].tid;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) dst[k * kThreads] = (addressable && pos[k] >= 0) ? (uint16_t)pos[k] : kNoSlot;
        }
    }
    if (l1.target != nullptr) {
        const float total = cta_sum(acc, reinterpret_cast<float *>(s_cc));
        if (threadIdx.x == 0) l1.partials[tile] = total;
    }
    if (pixel_topk != nullptr) {
        // the IDs by pixel into shared memory (positions read first, then overwritten), then each tile row of 16 pixels x 10 IDs (80
        // int2) written with consecutive threads
        int ids[kFwdPixels][kTopK];
#pragma unroll
        for (int q = 0; q < kFwdPixels; ++q)
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int position = s_ids[k * kThreads + pc[q].tid];
                ids[q][k] = position >= 0 ? __ldg(&ids_sorted[range.x + position]) : -1;
            }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < kFwdPixels; ++q)
#pragma unroll
            for (int k = 0; k < kTopK; ++k) s_ids[pc[q].tid * kTopK + k] = ids[q][k];
        __syncthreads();
        const int i0 = (tile / tiles_x) * kTile, j0 = (tile % tiles_x) * kTile;
        const int row_pairs = kTile * kTopK / 2;
        for (int idx = threadIdx.x; idx < kTile * row_pairs; idx += kFwdThreads) {
            const int ly = idx / row_pairs, rem = idx % row_pairs;
            const int lx = rem / (kTopK / 2), pair = rem % (kTopK / 2);
            const int i = i0 + ly, j = j0 + lx;
            if (i >= img_h || j >= img_w) continue;
            const int src = ((ly >> 2) * 2 + (lx >> 3)) * 32 + (ly & 3) * 8 + (lx & 7);
            const int2 v = make_int2(s_ids[src * kTopK + 2 * pair], s_ids[src * kTopK + 2 * pair + 1]);
            reinterpret_cast<int2 *>(pixel_topk)[((size_t)i * img_w + j) * (kTopK / 2) + pair] = v;
        }
    }
}

// Sum of NV values over the 32 lanes of a warp by recursive halving: at each step a lane keeps half of its values, adds the partner's
// copy of that half and hands over the other half, so NV - 1 + log2(32 / NV) shuffles replace 5 NV. Afterwards lane l holds the warp
// total of value index halving_index<NV>(l); lanes with l % (32 / NV) == 0 hold each index exactly once.
template <int NV>
__device__ __forceinline__ float warp_sum_scatter(float (&v)[NV], int lane) {
    int width = NV;
#pragma unroll
    for (int bit = 16; bit >= 32 / NV; bit >>= 1) {
        width >>= 1;
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int k = 0; k < NV / 2; ++k) {
            if (k < width) {
                const float keep = upper ? v[k + width] : v[k];
                const float give = upper ? v[k] : v[k + width];
                v[k] = keep + __shfl_xor_sync(0xffffffffu, give, bit);
            }
        }
    }
    float total = v[0];
#pragma unroll
    for (int bit = 16 / NV; bit >= 1; bit >>= 1) total += __shfl_xor_sync(0xffffffffu, total, bit);
    return total;
}

template <int NV>
__device__ __forceinline__ int halving_index(int lane) {
    int index = 0, width = NV;
#pragma unroll
    for (int bit = 16; bit >= 32 / NV; bit >>= 1) {
        width >>= 1;
        if (lane & bit) index += width;
    }
    return index;
}

// ---- backward pass of the [H, W, 10] operator --------------------------------------------------------------------------------------
//
// The operator's lists hold Gaussian IDs, with no tile list to index, so each warp (an 8x4 patch) walks the union of its pixels' IDs in
// increasing order (a warp-wide minimum per step); lanes whose pixel holds the current Gaussian contribute their values, the others
// zeros; the warp sums the 5 + C values (of two Gaussians at a time for C <= 3) with one recursive-halving reduce-scatter and one
// global atomic per value. Each pixel sorts its
// ten slots by ID once (a 29-comparator network on registers) and keeps them in shared memory, so that at every step of the walk its
// smallest unconsumed ID is at hand and its slot's values are two loads away, instead of a minimum and a select over ten registers.
// The few Gaussians of a warp's union are read through the L1 cache.
constexpr int kNoId = 0x7fffffff;

// A sorting network for 10 keys (29 comparators, depth 8), checked exhaustively on 0/1 inputs
__device__ __forceinline__ void sort10(int (&key)[kTopK]) {
    constexpr int kPairs[29][2] = {{4, 9}, {3, 8}, {2, 7}, {1, 6}, {0, 5}, {1, 4}, {6, 9}, {0, 3}, {5, 8}, {0, 2}, {3, 6}, {7, 9},
                                   {0, 1}, {2, 4}, {5, 7}, {8, 9}, {1, 2}, {4, 6}, {7, 8}, {3, 5}, {2, 5}, {6, 8}, {1, 3}, {4, 7},
                                   {2, 3}, {6, 7}, {3, 4}, {5, 6}, {4, 5}};
#pragma unroll
    for (int c = 0; c < 29; ++c) {
        const int i = kPairs[c][0], j = kPairs[c][1];
        const int lo = min(key[i], key[j]), hi = max(key[i], key[j]);
        key[i] = lo, key[j] = hi;
    }
}

// The slot key of the walk: the Gaussian ID above the slot index (4 bits), so that sorting keys orders the slots by ID; IDs below 2^27
constexpr int kSlotBits = 4;
constexpr int kMaxWalkId = (1 << (31 - kSlotBits)) - 1;

template <int C, int NV>
__global__ void __launch_bounds__(kThreads, NV <= 8 ? 5 : 3)
    raster_bwd_ids_kernel(const int tiles_x, const int img_h, const int img_w, const int channels_rt, const int num_points,
        const float2 *__restrict__ xys,
        const float *__restrict__ conics, const float *__restrict__ colors, const float *__restrict__ v_output,
        const int *__restrict__ pixel_topk, float *__restrict__ v_xy, float *__restrict__ v_conic, float *__restrict__ v_colors) {
    constexpr int kMaxC = C > 0 ? C : (NV - 5 < kMaxChannels ? NV - 5 : kMaxChannels);
    static_assert(5 + kMaxC <= NV, "NV must hold the 5 geometry values and the channels");
    const int channels = C > 0 ? C : channels_rt;
    const int lane = threadIdx.x & 31;
    const PixelCoord pc = tile_pixel(blockIdx.x, tiles_x, 0);
    const bool inside = pc.i < img_h && pc.j < img_w;
    const float px = (float)pc.j, py = (float)pc.i;
    const int num_pixels = img_h * img_w;
    const int p = inside ? pc.i * img_w + pc.j : 0;

    float v_out[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) v_out[c] = (inside && c < channels) ? __ldg(&v_output[(size_t)c * num_pixels + p]) : 0.f;
    int id[kTopK];
    float d[kTopK];
    float denom = (float)igs::kNormEps;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int id_in = inside ? __ldg(&pixel_topk[(size_t)p * kTopK + k]) : -1;
        const int g = id_in < num_points ? id_in : -1;  // an ID of N or more counts as an empty slot instead of reading out of bounds
        id[k] = g < 0 ? kNoId : g;
        d[k] = 0.f;
        if (g < 0) continue;
        const float2 xy = __ldg(&xys[g]);
        d[k] = __expf(-igs::gaussian_sigma(xy.x, xy.y, __ldg(&conics[3 * g]), __ldg(&conics[3 * g + 1]), __ldg(&conics[3 * g + 2]), px, py));
        denom += d[k];
    }
    // the reference's algebra with its divisions by denom as products with two reciprocals (fast-math division)
    const float inv = 1.f / denom, inv2 = 1.f / (denom * denom);
    float s[kTopK];
    float shared = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        s[k] = 0.f;
        if (id[k] == kNoId) continue;
#pragma unroll
        for (int c = 0; c < kMaxC; ++c)
            if (c < channels) s[k] += __ldg(&colors[(size_t)id[k] * channels + c]) * v_out[c];
        shared += -d[k] * inv2 * s[k];
    }
    // the pixel's slots in increasing ID order (empty slots, kNoId, last): keys (ID, slot) sorted in registers and kept in shared memory
    // with the slots' colour weight and dL/dsigma, so that each step of the walk finds the pixel's smallest unconsumed ID and its values
    // with a few loads
    __shared__ int s_key[kTopK][kThreads];
    __shared__ float2 s_wv[kTopK][kThreads];  // (colour weight, dL/dsigma)
    const int tid = threadIdx.x;
    int key[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        key[k] = id[k] == kNoId ? kNoId : (id[k] << kSlotBits) | k;
        s_wv[k][tid] = make_float2(d[k] * inv, -d[k] * (s[k] * inv + shared));
    }
    sort10(key);
#pragma unroll
    for (int k = 0; k < kTopK; ++k) s_key[k][tid] = key[k];

    // The walk. With NV <= 8 each step takes the two smallest IDs of the union and sums their 2 NV values in one reduce-scatter (fewer
    // shuffles and steps than one Gaussian at a time); wider value sets take one Gaussian per step.
    constexpr int kPerStep = NV <= 8 ? 2 : 1;
    constexpr int kValues = kPerStep * NV;
    const int index = halving_index<kValues>(lane);
    const int value_index = index % NV, which = index / NV;  // lane's value and its Gaussian of the step
    const bool adds = (lane % (32 / kValues)) == 0 && value_index < 5 + channels;
    float *const target = value_index < 3 ? v_conic + value_index : value_index < 5 ? v_xy + (value_index - 3) : v_colors + (value_index - 5);
    const int stride = value_index < 3 ? 3 : value_index < 5 ? 2 : channels;
    int pos = 0;
    int head = key[0];
    // the pixel's values for Gaussian cur (zero if it does not hold it); a pixel holding it moves to its next slot
    auto take = [&](const int cur, float &ws, float &vs) {
        ws = 0.f, vs = 0.f;
        if ((head >> kSlotBits) == cur) {
            const float2 wv = s_wv[head & ((1 << kSlotBits) - 1)][tid];
            ws = wv.x, vs = wv.y;
            ++pos;
            head = pos < kTopK ? s_key[pos][tid] : kNoId;
        }
    };
    auto values = [&](const int cur, const float ws, const float vs, float *val) {
        const float2 xy = __ldg(&xys[cur]);
        const float a = __ldg(&conics[3 * cur]), b = __ldg(&conics[3 * cur + 1]), c = __ldg(&conics[3 * cur + 2]);
        const float dx = xy.x - px, dy = xy.y - py;
        val[0] = vs * dx * dx;  // halved after the sum (exact: a power of two)
        val[1] = vs * dx * dy;
        val[2] = vs * dy * dy;
        val[3] = vs * (a * dx + b * dy);
        val[4] = vs * (b * dx + c * dy);
#pragma unroll
        for (int ch = 0; ch < NV - 5; ++ch) val[5 + ch] = ch < kMaxC ? ws * v_out[ch < kMaxC ? ch : 0] : 0.f;
    };
    int low = __reduce_min_sync(0xffffffffu, head);
    while (low != kNoId) {
        int cur[kPerStep];
        float ws[kPerStep], vs[kPerStep];
        bool valid[kPerStep];
#pragma unroll
        for (int q = 0; q < kPerStep; ++q) {
            valid[q] = low != kNoId;  // uniform over the warp; the first always is
            cur[q] = valid[q] ? low >> kSlotBits : cur[0];
            ws[q] = 0.f, vs[q] = 0.f;
            if (valid[q]) {
                take(cur[q], ws[q], vs[q]);
                low = __reduce_min_sync(0xffffffffu, head);
            }
        }
        float val[kValues];
#pragma unroll
        for (int q = 0; q < kPerStep; ++q) values(cur[q], ws[q], vs[q], val + q * NV);
        const float total = warp_sum_scatter<kValues>(val, lane);
        const bool last = which == kPerStep - 1;  // selects, not a dynamic index (which would put the arrays in local memory)
        if (adds && (last ? valid[kPerStep - 1] : valid[0]))
            atomicAdd(target + (size_t)stride * (last ? cur[kPerStep - 1] : cur[0]), (value_index == 0 || value_index == 2) ? 0.5f * total : total);
    }
}

// ---- backward pass from the tile lists, pairs grouped by Gaussian ---------------------------------------------------------------------
//
// The reference's per-pixel algebra (backward.cu:219-265): with D = 1e-4 + sum_k d_k, s_k = f_k . v_out and
// S = -sum_k d_k s_k / D^2, dL/dsigma_k = -d_k (s_k / D + S) and the colour weight is d_k / D. Since sum_k d_k s_k = v_out . U with
// U = sum_k d_k f_k (the unnormalised render), a pixel's pairs need only d_k, D, S and v_out: s_k is formed where the pair is summed,
// from the entry's colour, which is the same for every pair of that entry, so no per-pair gradient is stored. One CTA of 256 threads (one per pixel) per tile; lists longer than kPairStage entries go through steps 2-3
// in chunks of kPairStage:
//   1. per pixel: its slots' d_k (the selection's alphas, or exp(-sigma_k) recomputed from the tile lists) in shared memory, and its
//      coordinates, 1 / D, S and v_out;
//   2. the tile's (pixel, slot) pairs are grouped by list position with a counting sort in shared memory without atomics: per slot the
//      lanes of a warp holding the same entry are grouped (__match_any_sync) and the group's leader counts it in the warp's own row of
//      counters; a CTA-wide scan turns the (warp, entry) counts into places; each pair is stored at its place;
//   3. one warp per entry: the lanes stride over the entry's pairs (consecutive records are mostly consecutive pixels, so the shared
//      reads do not conflict), form v = dL/dsigma and w = d / D of each and sum v dx^2, v dx dy, v dy^2, v (a dx + b dy), v (b dx + c dy)
//      and w v_out (dx, dy from the Gaussian's center, a, b, c its conic), then one reduce-scatter over the warp and one global atomic per
//      value: v_conic = (S_xx / 2, S_xy, S_yy / 2), v_xy = the next two sums, v_color = S_c.
template <int kMaxC>
struct PairSmem {
    static constexpr bool kPackedOut = kMaxC <= 4;  // a pixel's v_out and an entry's features as one float4 each
    float4 geo[kPairStage];  // x, y, conic a / 2, conic b: per entry, or in pairs of entries (the selection's layout, stage_paired)
    float cc[kPairStage];    // conic c / 2
    float4 col4[kPackedOut ? kPairStage : 1];           // features (C <= 4, zero-padded)
    float col[kPackedOut ? 1 : kPairStage * kMaxC];      // features (C > 4)
    int gid[kPairStage];                                 // Gaussian IDs
    union {
        int pos[kTopK][kThreads];  // the selection's slots: positions in the tile's list (-1 empty), read into registers before step 2
        struct {
            uint16_t pairs[kPairs];                    // (slot << 8) | pixel, grouped by entry
            uint16_t wcnt[kThreads / 32][kPairStage];  // pairs per (warp, entry), then each warp's first place in the entry's segment
            int start[kPairStage + 1];                 // segment starts
        } g;
    };
    float alpha[kTopK][kThreads];                // d_k = exp(-sigma_k) of each slot (the selection's alphas)
    float4 pix[kThreads];                        // -x, -y, S
    float4 vout4[kPackedOut ? kThreads : 1];     // v_out / D (C <= 4)
    float vout[kPackedOut ? 1 : kMaxC][kPackedOut ? 1 : kThreads];  // v_out / D per channel (C > 4)
    int wsum[kThreads / 32];
};

// An entry's features into shared memory (zero beyond the channel count)
template <int kMaxC>
__device__ __forceinline__ void stage_colors(PairSmem<kMaxC> &sm, const int e, const float *__restrict__ f, const int channels) {
    if constexpr (PairSmem<kMaxC>::kPackedOut) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kMaxC; ++c)
            if (c < channels) v[c] = __ldg(&f[c]);
        sm.col4[e] = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int c = 0; c < kMaxC; ++c)
            if (c < channels) sm.col[e * kMaxC + c] = __ldg(&f[c]);
    }
}

// A staged entry's features (zero beyond the channel count)
template <int kMaxC>
__device__ __forceinline__ void staged_colors(const PairSmem<kMaxC> &sm, const int e, const int channels, float (&f)[kMaxC]) {
    if constexpr (PairSmem<kMaxC>::kPackedOut) {
        const float4 v = sm.col4[e];
        const float va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) f[c] = va[c];
    } else {
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) f[c] = c < channels ? sm.col[e * kMaxC + c] : 0.f;
    }
}

// Staged geometry of entry e, (x, y, a / 2, b), from either layout
template <bool kPaired>
__device__ __forceinline__ float4 staged_geo(const float4 *geo, const int e) {
    if constexpr (kPaired) return paired_geo(geo, e);
    else return geo[e];
}

// Stage entries [chunk, chunk + kPairStage) of a tile's list for the backward pass (every thread of the CTA calls it): centres, the conic
// halved as the selection stages it (a / 2, b, c / 2), per entry or in the selection's paired layout, and the colours
template <bool kPaired, int kMaxC>
__device__ __forceinline__ void stage_pair_chunk(PairSmem<kMaxC> &sm, const int chunk, const int len, const int2 range,
                                                 const int *__restrict__ ids_sorted, const float2 *__restrict__ xys,
                                                 const float *__restrict__ conics, const float *__restrict__ colors, const int channels) {
    const int n = min(kPairStage, len - chunk);
    for (int e = threadIdx.x; e < n; e += kThreads) {
        const int g = __ldg(&ids_sorted[range.x + chunk + e]);
        const float2 xy = __ldg(&xys[g]);
        sm.gid[e] = g;
        if constexpr (kPaired) {
            stage_paired(sm.geo, sm.cc, e, xy, __ldg(&conics[3 * g]), __ldg(&conics[3 * g + 1]), __ldg(&conics[3 * g + 2]));
        } else {
            sm.geo[e] = make_float4(xy.x, xy.y, 0.5f * __ldg(&conics[3 * g]), __ldg(&conics[3 * g + 1]));
            sm.cc[e] = 0.5f * __ldg(&conics[3 * g + 2]);
        }
        stage_colors(sm, e, colors + (size_t)g * channels, channels);
    }
}

// Step 1's per-pixel values: 1 / D and S = -sum_k d_k s_k / D^2 (s_k = f_k . v_out), formed as -(v_out . U) / D^2 from the pixel's
// U = sum_k d_k f_k: the same sum in another order (the reference adds the slots' terms, backward.cu:243-252), without reading the
// slots' features again. The reference's divisions by D and D^2 are products with approximate reciprocals under fast math; so are these.
template <int kMaxC>
__device__ __forceinline__ float2 pixel_terms(const float denom, const float (&u)[kMaxC], const float (&v_out)[kMaxC]) {
    const float inv = 1.f / denom, inv2 = 1.f / (denom * denom);
    float vu = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) vu = fmaf(v_out[c], u[c], vu);
    return make_float2(inv, -inv2 * vu);
}

// Step 1's per-pixel record: the negated coordinates, S and v_out / D (terms = (1 / D, S)). Step 3 forms dL/dsigma_k =
// -d_k (f_k . (v_out / D) + S) and the colour gradient d_k (v_out / D): the reference's -d_k (s_k / D + S) and (d_k / D) v_out with the
// division applied to v_out.
template <int kMaxC>
__device__ __forceinline__ void store_pixel_grad(PairSmem<kMaxC> &sm, const int tid, const float px, const float py, const float2 terms,
                                                 const float (&v_out)[kMaxC]) {
    sm.pix[tid] = make_float4(-px, -py, terms.y, 0.f);
    if constexpr (PairSmem<kMaxC>::kPackedOut) {
        float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) v4[c] = v_out[c] * terms.x;
        sm.vout4[tid] = make_float4(v4[0], v4[1], v4[2], v4[3]);
    } else {
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) sm.vout[c][tid] = v_out[c] * terms.x;
    }
}

// Transpose of a 32 x 32 bit matrix held one row per lane (bit j of lane l's word = M[l][j]): lane j returns column j (bit l = M[l][j]).
// Five exchanges of off-diagonal blocks between lanes l and l ^ s.
__device__ __forceinline__ unsigned transpose_bits(unsigned x, const int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const unsigned left = s == 16 ? 0x0000FFFFu : s == 8 ? 0x00FF00FFu : s == 4 ? 0x0F0F0F0Fu : s == 2 ? 0x33333333u : 0x55555555u;
        const unsigned y = __shfl_xor_sync(0xffffffffu, x, s);
        x = (lane & s) ? ((x & ~left) | ((y >> s) & left)) : ((x & left) | ((y << s) & ~left));
    }
    return x;
}

// Steps 2 and 3 of the pairs-grouped backward pass for one tile (every thread of the CTA calls it, after a CTA barrier that follows the
// last read of sm.pos): sm.alpha and sm.pix / sm.vout hold step 1's per-slot and per-pixel values, key[k] the list position of the
// thread's slot k (-1 empty). The staged chunk of the list is used for chunk 0 unless restage_first; every other chunk is staged by
// stage(chunk).
template <int NV, bool kPaired, int kMaxC, typename Stage>
__device__ __forceinline__ void pairs_grouped_sums(PairSmem<kMaxC> &sm, const int (&key)[kTopK], const int len, const int2 range,
                                                   const int *__restrict__ ids_sorted, const int channels, const bool restage_first,
                                                   Stage stage, float *__restrict__ v_xy, float *__restrict__ v_conic,
                                                   float *__restrict__ v_colors) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int value_index = halving_index<NV>(lane);
    const bool holds_total = (lane % (32 / NV)) == 0 && value_index < 5 + channels;
    for (int chunk = 0; chunk < len; chunk += kPairStage) {
        const int n_entries = min(kPairStage, len - chunk);
        if (chunk > 0 || restage_first) {
            __syncthreads();  // the previous chunk's pairs and parameters are consumed
            stage(chunk);
            __syncthreads();
        }
        // 2. counting sort of this chunk's pairs by entry without atomics. Each warp counts its pairs per entry in its own row of wcnt and
        //    gives each pair its place among the warp's pairs of that entry (< 32: 5 bits). A pixel holds an entry at most once, so for a
        //    chunk of at most 32 entries the warp's (lane, entry) incidence is a 32 x 32 bit matrix: transposed, lane e holds the lanes that
        //    hold entry e, whose count is the warp's count and among which a lane's rank is its place. Longer chunks group, per slot, the
        //    lanes holding the same entry with __match_any_sync, and the group's leader adds the group to the counter.
        const unsigned lanes_below = (1u << lane) - 1u;
        unsigned off_lo = 0u, off_hi = 0u;  // the pairs' places, 5 bits per slot
        if (n_entries <= 32) {
            unsigned held = 0u;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int e = key[k] - chunk;
                if (key[k] >= 0 && e >= 0 && e < n_entries) held |= 1u << e;
            }
            const unsigned holders = transpose_bits(held, lane);  // lanes holding entry `lane`
            if (lane < n_entries) sm.g.wcnt[warp][lane] = (uint16_t)__popc(holders);
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const unsigned of_entry = __shfl_sync(0xffffffffu, holders, (key[k] - chunk) & 31);
                const unsigned off = (unsigned)__popc(of_entry & lanes_below) & 31u;
                if (k < 6) off_lo |= off << (5 * k);
                else off_hi |= off << (5 * (k - 6));
            }
        } else {
            for (int e = lane; e < n_entries; e += 32) sm.g.wcnt[warp][e] = 0;
            __syncwarp();
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int e = key[k] - chunk;
                const bool mine = key[k] >= 0 && e >= 0 && e < n_entries;
                const unsigned peers = __match_any_sync(0xffffffffu, mine ? e : -1);
                const unsigned below = peers & lanes_below;
                const int base = mine ? (int)sm.g.wcnt[warp][e] : 0;
                __syncwarp();
                if (mine && below == 0u) sm.g.wcnt[warp][e] = (uint16_t)(base + __popc(peers));
                __syncwarp();
                const unsigned off = (unsigned)(base + __popc(below)) & 31u;
                if (k < 6) off_lo |= off << (5 * k);
                else off_hi |= off << (5 * (k - 6));
            }
        }
        __syncthreads();
        {
            // per entry (one thread each): the warps' counts into running places, the entry's total into a CTA-wide exclusive scan
            const int e = tid;
            int total = 0;
            if (e < n_entries) {
#pragma unroll
                for (int w = 0; w < kThreads / 32; ++w) {
                    const int c = sm.g.wcnt[w][e];
                    sm.g.wcnt[w][e] = (uint16_t)total;
                    total += c;
                }
            }
            int incl = total;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            if (lane == 31) sm.wsum[warp] = incl;
            __syncthreads();
            int before = 0;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) before += w < warp ? sm.wsum[w] : 0;
            const int start = before + incl - total;
            if (e < n_entries) {
                sm.g.start[e] = start;
#pragma unroll
                for (int w = 0; w < kThreads / 32; ++w) sm.g.wcnt[w][e] = (uint16_t)(sm.g.wcnt[w][e] + start);
            }
            if (e == n_entries - 1) sm.g.start[n_entries] = start + total;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            const int e = key[k] - chunk;
            const bool mine = key[k] >= 0 && e >= 0 && e < n_entries;
            const unsigned off = (k < 6 ? off_lo >> (5 * k) : off_hi >> (5 * (k - 6))) & 31u;
            if (mine) sm.g.pairs[sm.g.wcnt[warp][e] + off] = (uint16_t)((k << 8) | tid);
        }
        __syncthreads();

        // 3. one warp per entry. Packed instructions take two sums at a time: (dx, dy) = (x, y) + (-px, -py), (tx, ty) = v (dx, dy),
        //    (S_xx, S_xy) += tx (dx, dy), the two v_xy sums += (b, c) ty then (a, b) tx, and channel pairs += d (v_out / D); each component
        //    is rounded as the scalar fmaf / fadd / fmul would round it.
        for (int e = warp; e < n_entries; e += kThreads / 32) {
            const int b = sm.g.start[e], n = sm.g.start[e + 1] - b;
            if (n == 0) continue;  // no pixel kept this Gaussian (uniform over the warp)
            const float4 q = staged_geo<kPaired>(sm.geo, e);
            const float ca = 2.f * q.z, cb = q.w, cc = 2.f * sm.cc[e];  // the staged conic is halved; doubling it back is exact
            const float2 qxy = make_float2(q.x, q.y), cbc = make_float2(cb, cc), cab = make_float2(ca, cb);
            float f[kMaxC];
            staged_colors(sm, e, channels, f);
            float2 s01 = make_float2(0.f, 0.f), s34 = make_float2(0.f, 0.f);
            float s2 = 0.f;
            float sc[kMaxC];
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) sc[c] = 0.f;
            for (int i = lane; i < n; i += 32) {
                const unsigned rec = sm.g.pairs[b + i];
                const int slot = (int)(rec >> 8), pix = (int)(rec & 255u);
                const float d = sm.alpha[slot][pix];
                const float4 pr = sm.pix[pix];  // -x, -y, S
                float vo[kMaxC];                 // v_out / D
                if constexpr (PairSmem<kMaxC>::kPackedOut) {
                    const float4 v4 = sm.vout4[pix];
                    const float va[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                    for (int c = 0; c < kMaxC; ++c) vo[c] = va[c];
                } else {
#pragma unroll
                    for (int c = 0; c < kMaxC; ++c) vo[c] = c < channels ? sm.vout[c][pix] : 0.f;
                }
                float sk = 0.f;  // f_k . v_out / D in the reference's channel order
#pragma unroll
                for (int c = 0; c < kMaxC; ++c) sk = fmaf(f[c], vo[c], sk);
                const float vs = -d * (sk + pr.z);  // dL/dsigma
                const float2 dxy = __fadd2_rn(qxy, make_float2(pr.x, pr.y));
                const float2 t = __fmul2_rn(make_float2(vs, vs), dxy);
                s01 = __ffma2_rn(make_float2(t.x, t.x), dxy, s01);
                s2 = fmaf(t.y, dxy.y, s2);
                // v_xy per pair, a v dx + b v dy and b v dx + c v dy, as the reference sums v (a dx + b dy): with the conic factored out of
                // the sums, a Sx and b Sy can cancel to a few parts in 10^4 of themselves and lose the result's accuracy
                s34 = __ffma2_rn(cbc, make_float2(t.y, t.y), s34);
                s34 = __ffma2_rn(cab, make_float2(t.x, t.x), s34);
                add_weighted(d, vo, sc);
            }
            float acc[NV];
            acc[0] = s01.x, acc[1] = s01.y, acc[2] = s2, acc[3] = s34.x, acc[4] = s34.y;
#pragma unroll
            for (int v = 5; v < NV; ++v) acc[v] = v - 5 < kMaxC && v - 5 < channels ? sc[v - 5 < kMaxC ? v - 5 : 0] : 0.f;
            const float total = warp_sum_scatter<NV>(acc, lane);
            if (holds_total) {
                // the gradient value this lane adds: v_conic (S_xx / 2, S_xy, S_yy / 2), v_xy, v_colors
                const int g = sm.gid[e];
                float *const target = value_index < 3 ? v_conic + 3 * (size_t)g + value_index
                                    : value_index < 5 ? v_xy + 2 * (size_t)g + (value_index - 3)
                                                      : v_colors + (size_t)g * channels + (value_index - 5);
                const float value = (value_index == 0 || value_index == 2) ? 0.5f * total : total;
                if (value != 0.f) atomicAdd(target, value);
            }
        }
    }
}

template <int C, int NV>
__global__ void __launch_bounds__(kThreads, NV > 8 ? 3 : C > 0 ? 5 : 4)
    raster_bwd_pairs_kernel(const int tiles_x, const int img_h, const int img_w, const int row_begin, const int band_h,
        const int channels_rt, const int *__restrict__ ids_sorted, const int2 *__restrict__ tile_bins, const float2 *__restrict__ xys,
        const float *__restrict__ conics, const float *__restrict__ colors, const float *__restrict__ v_output,
        const uint16_t *__restrict__ tile_topk, float *__restrict__ v_xy, float *__restrict__ v_conic, float *__restrict__ v_colors) {
    igs::wait_for_predecessor();
    constexpr int kMaxC = C > 0 ? C : (NV - 5 < kMaxChannels ? NV - 5 : kMaxChannels);
    static_assert(5 + kMaxC <= NV, "NV must hold the 5 geometry sums and the channels");
    const int channels = C > 0 ? C : channels_rt;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PairSmem<kMaxC> &sm = *reinterpret_cast<PairSmem<kMaxC> *>(smem_raw);

    const int tile = blockIdx.x;
    const int2 range = tile_bins[tile];
    const int len = range.y - range.x;
    if (len <= 0) return;
    const int tid = threadIdx.x;
    const PixelCoord pc = tile_pixel(tile, tiles_x, row_begin);
    const bool inside = pc.i < img_h && pc.j < img_w;
    const float px = (float)pc.j, py = (float)pc.i;
    const int num_pixels = band_h * img_w;  // one channel plane of the (band of the) image
    const int p = inside ? (pc.i - row_begin * kTile) * img_w + pc.j : 0;

    // the pixel's loads, issued before the staging barrier so that their latency overlaps it
    float v_out[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) v_out[c] = (inside && c < channels) ? __ldg(&v_output[(size_t)c * num_pixels + p]) : 0.f;
    int key[kTopK];
    if (len < (int)kNoSlot) {
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            // empty (kNoSlot) or, in lists not written by the forward pass, past the end of the list: no entry
            const uint16_t v = inside ? __ldg(&tile_topk[((size_t)tile * kTopK + k) * kThreads + tid]) : kNoSlot;
            key[k] = (int)v < len ? (int)v : -1;
        }
    } else {
        // a list too long for 16-bit positions: select the pixel's top-K again, exactly as the forward pass did
        const PixelCoord pcs[1] = {pc};
        const bool ins[1] = {inside};
        float val[1][kTopK];
        select_topk<1>(range, ids_sorted, xys, conics, pcs, ins, sm.geo, sm.cc, &sm.pos[0][0], &sm.alpha[0][0], val);
#pragma unroll
        for (int k = 0; k < kTopK; ++k) key[k] = sm.pos[k][tid];
        __syncthreads();  // the staging arrays and the positions (sm.pos, shared with step 2's arrays) are reused below
    }

    // stage the first chunk of the list (lists longer than kPairStage are processed in chunks; their other entries are read from global
    // memory in step 1)
    auto stage = [&](int chunk) { stage_pair_chunk<false>(sm, chunk, len, range, ids_sorted, xys, conics, colors, channels); };
    stage(0);
    __syncthreads();

    // 1. the slots' d_k = exp(-sigma_k) (the reference's sigma, forward.cu:309-311) and the pixel's record
    float denom = (float)igs::kNormEps;
    float u[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) u[c] = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        float d = 0.f;
        if (key[k] >= 0) {
            if (key[k] < kPairStage) {
                const int e = key[k];
                d = __expf(-halved_sigma(sm.geo[e], sm.cc[e], px, py));
                float f[kMaxC];
                staged_colors(sm, e, channels, f);
                add_weighted(d, f, u);
            } else {
                // past the staged chunk of a longer list
                const int g = __ldg(&ids_sorted[range.x + key[k]]);
                const float2 xy = __ldg(&xys[g]);
                d = __expf(-igs::gaussian_sigma(xy.x, xy.y, __ldg(&conics[3 * g]), __ldg(&conics[3 * g + 1]), __ldg(&conics[3 * g + 2]), px,
                                                py));
#pragma unroll
                for (int c = 0; c < kMaxC; ++c)
                    if (c < channels) u[c] = fmaf(d, __ldg(&colors[(size_t)g * channels + c]), u[c]);
            }
            denom += d;
        }
        sm.alpha[k][tid] = d;
    }
    store_pixel_grad(sm, tid, px, py, pixel_terms<kMaxC>(denom, u, v_out), v_out);

    pairs_grouped_sums<NV, false>(sm, key, len, range, ids_sorted, channels, false, stage, v_xy, v_conic, v_colors);
}

// ---- the training step's rasterization in one kernel -------------------------------------------------------------------------------
//
// With the L1 loss, the gradient with respect to the image, sign(image - target) * ratio / numel, is known as soon as a pixel's value is.
// So one CTA per tile (256 threads, one pixel each) runs the forward and the backward pass of its tile back to back:
//   * the top-K selection (select_topk, slots in sm.pos / sm.alpha), the normalized sum U / D, the image, the tile's part of the loss
//     and the pixel's loss gradient;
//   * the backward's step 1 from the selection's alphas (the backward pass recomputes the same alphas bit for bit, so they stay in
//     shared memory) and the render's U, then steps 2 and 3 (pairs_grouped_sums) on the list still staged in shared memory.
// Neither the top-K lists nor the image gradient go through HBM, and each slot's alpha and colour are read once for the render.
template <int C, int NV>
__global__ void __launch_bounds__(kThreads, NV > 8 ? 3 : C > 0 ? 5 : 4)
    raster_step_kernel(const int tiles_x, const int img_h, const int img_w, const int row_begin, const int band_h, const int channels_rt,
        const int *__restrict__ ids_sorted, const int2 *__restrict__ tile_bins, const float2 *__restrict__ xys,
        const float *__restrict__ conics, const float *__restrict__ colors, const FusedL1 l1, float *__restrict__ out_img,
        float *__restrict__ v_xy, float *__restrict__ v_conic, float *__restrict__ v_colors) {
    igs::wait_for_predecessor();
    constexpr int kMaxC = C > 0 ? C : (NV - 5 < kMaxChannels ? NV - 5 : kMaxChannels);
    static_assert(5 + kMaxC <= NV, "NV must hold the 5 geometry sums and the channels");
    const int channels = C > 0 ? C : channels_rt;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PairSmem<kMaxC> &sm = *reinterpret_cast<PairSmem<kMaxC> *>(smem_raw);

    const int tile = blockIdx.x;
    const int2 range = tile_bins[tile];
    const int len = range.y - range.x;
    const int tid = threadIdx.x;
    const PixelCoord pc = tile_pixel(tile, tiles_x, row_begin);
    const bool inside = pc.i < img_h && pc.j < img_w;
    const int num_pixels = band_h * img_w;  // one channel plane of the (band of the) image
    const int p = inside ? (pc.i - row_begin * kTile) * img_w + pc.j : 0;

    // 1. forward: the top-K selection; a one-chunk list keeps its staged geometry and gets its colours staged beside it
    const PixelCoord pcs[1] = {pc};
    const bool ins[1] = {inside};
    float val[1][kTopK];
    select_topk<1>(range, ids_sorted, xys, conics, pcs, ins, sm.geo, sm.cc, &sm.pos[0][0], &sm.alpha[0][0], val);
    int key[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) key[k] = sm.pos[k][tid];
    const bool one_chunk = len <= kPairStage;
    if (one_chunk) {
        for (int e = tid; e < len; e += kThreads) {
            const int g = __ldg(&ids_sorted[range.x + e]);
            sm.gid[e] = g;
            stage_colors(sm, e, colors + (size_t)g * channels, channels);
        }
    }
    __syncthreads();  // the colours are staged, and every slot position is read (sm.pos is step 2's space)

    // 2. the pixel's value U / D (U = sum_k d_k f_k in slot order, D = 1e-4 + sum_k d_k), the image, the L1 loss and its gradient
    float target[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) target[c] = (inside && c < channels) ? __ldcs(&l1.target[(size_t)c * num_pixels + p]) : 0.f;
    float denom = (float)igs::kNormEps;
    float u[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) u[c] = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        if (key[k] < 0) continue;
        const float d = val[0][k];
        denom += d;
        float f[kMaxC];
        if (one_chunk) {
            staged_colors(sm, key[k], channels, f);
        } else {
            const float *fg = colors + (size_t)__ldg(&ids_sorted[range.x + key[k]]) * channels;
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) f[c] = c < channels ? __ldg(&fg[c]) : 0.f;
        }
        add_weighted(d, f, u);
    }
    const float inv_denom = 1.f / denom;
    float v_out[kMaxC];
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        v_out[c] = 0.f;
        if (!inside || c >= channels) continue;
        const float pix = u[c] * inv_denom;
        out_img[(size_t)c * num_pixels + p] = pix;
        const float d = pix - target[c];
        acc += fabsf(d);
        v_out[c] = l1_sign(d) * l1.grad_value;
        if (l1.v_output != nullptr) __stcs(&l1.v_output[(size_t)c * num_pixels + p], v_out[c]);
    }
    const float total = cta_sum(acc, reinterpret_cast<float *>(sm.wsum));
    if (tid == 0) l1.partials[tile] = total;
    if (len <= 0) return;

    // 3. backward, step 1: the pixel's record (the slots' d_k are the selection's alphas, in sm.alpha)
    const float2 terms = pixel_terms<kMaxC>(denom, u, v_out);
    store_pixel_grad(sm, tid, (float)pc.j, (float)pc.i, terms, v_out);

    // 4. backward, steps 2 and 3
    auto stage = [&](int chunk) { stage_pair_chunk<true>(sm, chunk, len, range, ids_sorted, xys, conics, colors, channels); };
    pairs_grouped_sums<NV, true>(sm, key, len, range, ids_sorted, channels, !one_chunk, stage, v_xy, v_conic, v_colors);
}

template <int C, int NV>
cudaError_t launch_step(int tiles, int tiles_x, int img_h, int img_w, int row_begin, int band_h, int channels, const int *ids,
                        const int2 *bins, const float2 *xys, const float *conics, const float *colors, const FusedL1 &l1, float *out_img,
                        float *v_xy, float *v_conic, float *v_colors, cudaStream_t s) {
    constexpr int kMaxC = C > 0 ? C : (NV - 5 < kMaxChannels ? NV - 5 : kMaxChannels);
    const size_t bytes = sizeof(PairSmem<kMaxC>);
    cudaError_t err = cudaFuncSetAttribute(raster_step_kernel<C, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err != cudaSuccess) return err;
    return igs::launch(raster_step_kernel<C, NV>, tiles, kThreads, bytes, s, tiles_x, img_h, img_w, row_begin, band_h, channels, ids, bins,
                       xys, conics, colors, l1, out_img, v_xy, v_conic, v_colors);
}

template <int C>
cudaError_t launch_fwd(int tiles, int tiles_x, int img_h, int img_w, int row_begin, int band_h, int channels, const int *ids, const int2 *bins,
                       const float2 *xys, const float *conics, const float *colors, float *out, int *pixel_topk, uint16_t *tile_topk,
                       const FusedL1 &l1, cudaStream_t s) {
    return igs::launch(raster_fwd_kernel<C>, tiles, kFwdThreads, 0, s, tiles_x, img_h, img_w, row_begin, band_h, channels, ids, bins, xys,
                       conics, colors, out, pixel_topk, tile_topk, l1);
}

int raster_fwd(int tiles_x, int tiles_y, int img_h, int img_w, int row_begin, int row_end, int channels, const int32_t *ids_sorted,
               const int32_t *tile_bins, const float *xys, const float *conics, const float *colors, float *out_img, int32_t *pixel_topk,
               uint16_t *tile_topk, void *stream, const char *who, FusedL1 l1 = FusedL1{}) {
    IGS_REQUIRE(tiles_x >= 0 && tiles_y >= 0 && img_h >= 0 && img_w >= 0, "%s: negative size", who);
    IGS_REQUIRE(channels >= 0 && channels <= kMaxChannels, "%s: at most %d channels (got %d)", who, kMaxChannels, channels);
    IGS_REQUIRE(tiles_x == igs::ceil_div(img_w, kTile) && tiles_y == igs::ceil_div(img_h, kTile),
                "%s: tile grid %dx%d does not cover a %dx%d image with %dx%d tiles", who, tiles_x, tiles_y, img_w, img_h, kTile, kTile);
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "%s: tile rows [%d, %d) outside [0, %d)", who, row_begin,
                row_end, tiles_y);
    IGS_REQUIRE(pixel_topk == nullptr || (row_begin == 0 && row_end == tiles_y), "%s: [H, W, 10] lists cover the whole image", who);
    const int tiles = tiles_x * (row_end - row_begin);
    if (tiles == 0) return IGS_OK;
    const int band_h = std::min(img_h, row_end * kTile) - row_begin * kTile;
    IGS_REQUIRE(tile_bins && xys && conics && (colors || channels == 0) && (out_img || channels == 0), "%s: null pointer", who);
    IGS_REQUIRE(igs::aligned(tile_bins, 8) && igs::aligned(xys, 8), "%s: tile_bins and xys must be 8-byte aligned", who);
    IGS_REQUIRE(pixel_topk == nullptr || igs::aligned(pixel_topk, 8), "%s: pixel_topk must be 8-byte aligned", who);
    cudaStream_t s = igs::as_stream(stream);
    const int2 *bins = reinterpret_cast<const int2 *>(tile_bins);
    const float2 *xy2 = reinterpret_cast<const float2 *>(xys);
    // channel counts with a specialised kernel, else the generic one
    const auto launch = channels == 1 ? launch_fwd<1> : channels == 3 ? launch_fwd<3> : channels == 9 ? launch_fwd<9> : launch_fwd<0>;
    const cudaError_t err = launch(tiles, tiles_x, img_h, img_w, row_begin, band_h, channels, ids_sorted, bins, xy2, conics, colors, out_img,
                                   pixel_topk, tile_topk, l1, s);
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
    return IGS_OK;
}

template <int C, int NV>
cudaError_t launch_bwd_ids(int tiles, int tiles_x, int img_h, int img_w, int channels, int num_points, const float2 *xys, const float *conics,
                           const float *colors, const float *v_output, const int *pixel_topk, float *v_xy, float *v_conic, float *v_colors,
                           cudaStream_t s) {
    return igs::launch(raster_bwd_ids_kernel<C, NV>, tiles, kThreads, 0, s, tiles_x, img_h, img_w, channels, num_points, xys, conics,
                       colors, v_output, pixel_topk, v_xy, v_conic, v_colors);
}

template <int C, int NV>
cudaError_t launch_bwd_pairs(int tiles, int tiles_x, int img_h, int img_w, int row_begin, int band_h, int channels, const int *ids,
                             const int2 *bins, const float2 *xys, const float *conics, const float *colors, const float *v_output,
                             const uint16_t *tile_topk, float *v_xy, float *v_conic, float *v_colors, cudaStream_t s) {
    constexpr int kMaxC = C > 0 ? C : (NV - 5 < kMaxChannels ? NV - 5 : kMaxChannels);
    const size_t bytes = sizeof(PairSmem<kMaxC>);
    // more than the 48 KB default of dynamic shared memory (set on every call: cheap, and correct for whichever device is current)
    cudaError_t err = cudaFuncSetAttribute(raster_bwd_pairs_kernel<C, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err != cudaSuccess) return err;
    return igs::launch(raster_bwd_pairs_kernel<C, NV>, tiles, kThreads, bytes, s, tiles_x, img_h, img_w, row_begin, band_h, channels, ids,
                       bins, xys, conics, colors, v_output, tile_topk, v_xy, v_conic, v_colors);
}

// The backward kernels accumulate with atomics: zero the gradients first, with one memset when v_xy, v_conic and v_colors are one block
cudaError_t zero_gradients(int num_points, int channels, float *v_xy, float *v_conic, float *v_colors, cudaStream_t s) {
    const size_t n = (size_t)num_points;
    if (v_conic == v_xy + 2 * n && (channels == 0 || v_colors == v_conic + 3 * n))
        return cudaMemsetAsync(v_xy, 0, sizeof(float) * (5 + (size_t)channels) * n, s);
    cudaError_t e = cudaMemsetAsync(v_xy, 0, sizeof(float) * 2 * n, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(v_conic, 0, sizeof(float) * 3 * n, s);
    if (e == cudaSuccess && channels > 0) e = cudaMemsetAsync(v_colors, 0, sizeof(float) * (size_t)channels * n, s);
    return e;
}

int raster_bwd(int img_h, int img_w, int row_begin, int row_end, int channels, int num_points, const int32_t *ids_sorted,
               const int32_t *tile_bins, const float *xys,
               const float *conics, const float *colors, const float *v_output, const int32_t *pixel_topk, const uint16_t *tile_topk,
               float *v_xy, float *v_conic, float *v_colors, void *stream, const char *who) {
    IGS_REQUIRE(img_h >= 0 && img_w >= 0 && num_points >= 0, "%s: negative size", who);
    IGS_REQUIRE(channels >= 0 && channels <= kMaxChannels, "%s: at most %d channels (got %d)", who, kMaxChannels, channels);
    cudaStream_t s = igs::as_stream(stream);
    if (num_points > 0) {
        IGS_REQUIRE(v_xy && v_conic && (v_colors || channels == 0), "%s: null gradient pointer", who);
        if (zero_gradients(num_points, channels, v_xy, v_conic, v_colors, s) != cudaSuccess) return igs::check_launch(who);
    }
    const int tiles_x = igs::ceil_div(img_w, kTile), tiles_y = igs::ceil_div(img_h, kTile);
    if (row_end < 0) row_end = tiles_y;
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "%s: tile rows [%d, %d) outside [0, %d)", who, row_begin,
                row_end, tiles_y);
    IGS_REQUIRE(pixel_topk == nullptr || (row_begin == 0 && row_end == tiles_y), "%s: [H, W, 10] lists cover the whole image", who);
    const int tiles = tiles_x * (row_end - row_begin);
    const int band_h = std::min(img_h, row_end * kTile) - row_begin * kTile;
    if (tiles == 0 || num_points == 0) return IGS_OK;
    IGS_REQUIRE(xys && conics && (colors || channels == 0) && (v_output || channels == 0), "%s: null pointer", who);
    IGS_REQUIRE(pixel_topk || (tile_topk && tile_bins && ids_sorted), "%s: null top-K lists", who);
    IGS_REQUIRE(pixel_topk == nullptr || num_points <= kMaxWalkId + 1, "%s: at most %d Gaussians with [H, W, 10] lists", who,
                kMaxWalkId + 1);
    IGS_REQUIRE(igs::aligned(xys, 8), "%s: xys must be 8-byte aligned", who);
    const int2 *bins = reinterpret_cast<const int2 *>(tile_bins);
    const float2 *xy2 = reinterpret_cast<const float2 *>(xys);
    // specialised kernels for 3 and 9 channels; otherwise the generic kernel with room for 5 + C sums (NV of 8, 16 or 32)
    cudaError_t err;
    if (tile_topk != nullptr) {
        const auto launch = channels == 3    ? launch_bwd_pairs<3, 8>
                            : channels <= 3  ? launch_bwd_pairs<0, 8>
                            : channels == 9  ? launch_bwd_pairs<9, 16>
                            : channels <= 11 ? launch_bwd_pairs<0, 16>
                                             : launch_bwd_pairs<0, 32>;
        err = launch(tiles, tiles_x, img_h, img_w, row_begin, band_h, channels, ids_sorted, bins, xy2, conics, colors, v_output, tile_topk,
                     v_xy, v_conic, v_colors, s);
    } else {
        const auto launch = channels == 3    ? launch_bwd_ids<3, 8>
                            : channels <= 3  ? launch_bwd_ids<0, 8>
                            : channels == 9  ? launch_bwd_ids<9, 16>
                            : channels <= 11 ? launch_bwd_ids<0, 16>
                                             : launch_bwd_ids<0, 32>;
        err = launch(tiles, tiles_x, img_h, img_w, channels, num_points, xy2, conics, colors, v_output, pixel_topk, v_xy, v_conic, v_colors,
                     s);
    }
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
    return IGS_OK;
}

// The fused training step over tile rows [row_begin, row_end) (the whole image: 0, tiles_y): image, loss, gradients
int raster_step(int tiles_x, int tiles_y, int img_h, int img_w, int row_begin, int row_end, int channels, int num_points,
                const int32_t *ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics, const float *colors,
                const float *target, float ratio, float *out_img, float *loss, float *v_output, float *v_xy, float *v_conic, float *v_colors,
                void *workspace, size_t workspace_bytes, void *stream, const char *who, bool gradients_zeroed = false,
                bool finish_loss = true) {
    IGS_REQUIRE(tiles_x >= 0 && tiles_y >= 0 && img_h >= 0 && img_w >= 0 && num_points >= 0, "%s: negative size", who);
    IGS_REQUIRE(channels >= 1 && channels <= kMaxChannels, "%s: 1 to %d channels (got %d)", who, kMaxChannels, channels);
    IGS_REQUIRE(tiles_x == igs::ceil_div(img_w, kTile) && tiles_y == igs::ceil_div(img_h, kTile),
                "%s: tile grid %dx%d does not cover a %dx%d image with %dx%d tiles", who, tiles_x, tiles_y, img_w, img_h, kTile, kTile);
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "%s: tile rows [%d, %d) outside [0, %d)", who, row_begin,
                row_end, tiles_y);
    const int tiles = tiles_x * (row_end - row_begin);
    IGS_REQUIRE(loss != nullptr || !finish_loss, "%s: null loss", who);
    IGS_REQUIRE(num_points == 0 || (v_xy && v_conic && v_colors), "%s: null gradient pointer", who);
    cudaStream_t s = igs::as_stream(stream);
    if (num_points > 0 && !gradients_zeroed && zero_gradients(num_points, channels, v_xy, v_conic, v_colors, s) != cudaSuccess)
        return igs::check_launch(who);
    if (tiles == 0) {  // no pixels (an empty band): no loss, zero gradients
        if (finish_loss && cudaMemsetAsync(loss, 0, sizeof(float), s) != cudaSuccess) return igs::check_launch(who);
        return IGS_OK;
    }
    IGS_REQUIRE(tile_bins && target && out_img && workspace, "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || (ids_sorted && xys && conics && colors), "%s: null Gaussian pointer", who);  // unread without Gaussians
    IGS_REQUIRE(igs::aligned(tile_bins, 8) && igs::aligned(xys, 8), "%s: tile_bins and xys must be 8-byte aligned", who);
    IGS_REQUIRE(workspace_bytes >= igs_raster_l1_workspace(tiles), "%s: workspace too small (%zu bytes, need %zu)", who, workspace_bytes,
                igs_raster_l1_workspace(tiles));
    IGS_REQUIRE(igs::aligned(workspace, 16), "%s: workspace must be 16-byte aligned", who);
    const float numel = (float)((int64_t)channels * img_h * img_w);
    FusedL1 l1;
    l1.target = target;
    l1.v_output = v_output;
    l1.grad_value = ratio / numel;
    l1.partials = static_cast<float *>(workspace);
    const int band_h = std::min(img_h, row_end * kTile) - row_begin * kTile;
    const auto launch = channels == 3    ? launch_step<3, 8>
                        : channels <= 3  ? launch_step<0, 8>
                        : channels == 9  ? launch_step<9, 16>
                        : channels <= 11 ? launch_step<0, 16>
                                         : launch_step<0, 32>;
    const cudaError_t err = launch(tiles, tiles_x, img_h, img_w, row_begin, band_h, channels, ids_sorted,
                                   reinterpret_cast<const int2 *>(tile_bins), reinterpret_cast<const float2 *>(xys), conics, colors, l1,
                                   out_img, v_xy, v_conic, v_colors, s);
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
    if (finish_loss) igs::launch(l1_finish_kernel, 1, kFinishThreads, 0, s, l1.partials, tiles, ratio, numel, loss);
    return igs::check_launch(who);
}

}  // namespace

extern "C" {

int igs_raster_fwd_topk(int tiles_x, int tiles_y, int img_height, int img_width, int channels, const int32_t *gaussian_ids_sorted,
                        const int32_t *tile_bins, const float *xys, const float *conics, const float *colors, float *out_img,
                        int32_t *pixel_topk, void *stream) {
    IGS_REQUIRE(pixel_topk != nullptr || (int64_t)img_height * img_width == 0, "igs_raster_fwd_topk: null pixel_topk");
    return raster_fwd(tiles_x, tiles_y, img_height, img_width, 0, tiles_y, channels, gaussian_ids_sorted, tile_bins, xys, conics, colors,
                      out_img, pixel_topk, nullptr, stream, "igs_raster_fwd_topk");
}

int igs_raster_fwd_topk_tiles(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int max_list_len,
                              const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                              const float *colors, float *out_img, uint16_t *tile_topk, void *stream) {
    IGS_REQUIRE(tile_topk != nullptr || tiles_x * tiles_y == 0, "igs_raster_fwd_topk_tiles: null tile_topk");
    IGS_REQUIRE(max_list_len >= 0, "igs_raster_fwd_topk_tiles: negative max_list_len");
    return raster_fwd(tiles_x, tiles_y, img_height, img_width, 0, tiles_y, channels, gaussian_ids_sorted, tile_bins, xys, conics, colors,
                      out_img, nullptr, tile_topk, stream, "igs_raster_fwd_topk_tiles");
}

int igs_raster_bwd_topk(int img_height, int img_width, int channels, int num_points, const float *xys, const float *conics,
                        const float *colors, const float *v_output, const int32_t *pixel_topk, float *v_xy, float *v_conic,
                        float *v_colors, void *stream) {
    return raster_bwd(img_height, img_width, 0, -1, channels, num_points, nullptr, nullptr, xys, conics, colors, v_output, pixel_topk, nullptr,
                      v_xy, v_conic, v_colors, stream, "igs_raster_bwd_topk");
}

int igs_raster_bwd_topk_tiles(int img_height, int img_width, int channels, int num_points, const int32_t *gaussian_ids_sorted,
                              const int32_t *tile_bins, const float *xys, const float *conics, const float *colors, const float *v_output,
                              const uint16_t *tile_topk, float *v_xy, float *v_conic, float *v_colors, void *stream) {
    IGS_REQUIRE(tile_topk != nullptr, "igs_raster_bwd_topk_tiles: null tile_topk");
    return raster_bwd(img_height, img_width, 0, -1, channels, num_points, gaussian_ids_sorted, tile_bins, xys, conics, colors, v_output, nullptr,
                      tile_topk, v_xy, v_conic, v_colors, stream, "igs_raster_bwd_topk_tiles");
}

int igs_raster_fwd_topk_tiles_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                                   int max_list_len, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                                   const float *conics, const float *colors, float *out_band, uint16_t *tile_topk, void *stream) {
    IGS_REQUIRE(max_list_len >= 0, "igs_raster_fwd_topk_tiles_band: negative max_list_len");
    IGS_REQUIRE(tile_topk != nullptr || row_begin == row_end, "igs_raster_fwd_topk_tiles_band: null tile_topk");
    return raster_fwd(tiles_x, tiles_y, img_height, img_width, row_begin, row_end, channels, gaussian_ids_sorted, tile_bins, xys, conics,
                      colors, out_band, nullptr, tile_topk, stream, "igs_raster_fwd_topk_tiles_band");
}

size_t igs_raster_l1_workspace(int num_tiles) { return sizeof(float) * (size_t)(num_tiles > 0 ? num_tiles : 1); }

int igs_raster_fwd_topk_tiles_l1_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                                      int max_list_len, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                                      const float *conics, const float *colors, const float *target, float ratio, float *out_img,
                                      uint16_t *tile_topk, float *loss, float *v_output, void *workspace, size_t workspace_bytes,
                                      void *stream) {
    const char *who = "igs_raster_fwd_topk_tiles_l1";
    IGS_REQUIRE(max_list_len >= 0, "%s: negative max_list_len", who);
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y && tiles_x >= 0, "%s: bad tile rows", who);
    const int tiles = tiles_x * (row_end - row_begin);
    if (tiles == 0) return IGS_OK;
    IGS_REQUIRE(channels >= 1, "%s: the loss needs at least one channel", who);
    IGS_REQUIRE(tile_topk && target && loss && v_output && workspace, "%s: null pointer", who);
    IGS_REQUIRE(workspace_bytes >= igs_raster_l1_workspace(tiles), "%s: workspace too small (%zu bytes, need %zu)", who, workspace_bytes,
                igs_raster_l1_workspace(tiles));
    IGS_REQUIRE(igs::aligned(workspace, 16), "%s: workspace must be 16-byte aligned", who);
    const float numel = (float)((int64_t)channels * img_height * img_width);
    FusedL1 l1;
    l1.target = target;
    l1.v_output = v_output;
    l1.grad_value = ratio / numel;
    l1.partials = static_cast<float *>(workspace);
    const int status = raster_fwd(tiles_x, tiles_y, img_height, img_width, row_begin, row_end, channels, gaussian_ids_sorted, tile_bins, xys,
                                  conics, colors, out_img, nullptr, tile_topk, stream, who, l1);
    if (status != IGS_OK) return status;
    igs::launch(l1_finish_kernel, 1, kFinishThreads, 0, igs::as_stream(stream), l1.partials, tiles, ratio, numel, loss);
    return igs::check_launch(who);
}

int igs_raster_fwd_topk_tiles_l1(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int max_list_len,
                                 const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                                 const float *colors, const float *target, float ratio, float *out_img, uint16_t *tile_topk, float *loss,
                                 float *v_output, void *workspace, size_t workspace_bytes, void *stream) {
    return igs_raster_fwd_topk_tiles_l1_band(tiles_x, tiles_y, img_height, img_width, 0, tiles_y, channels, max_list_len,
                                             gaussian_ids_sorted, tile_bins, xys, conics, colors, target, ratio, out_img, tile_topk, loss,
                                             v_output, workspace, workspace_bytes, stream);
}

int igs_raster_bwd_topk_tiles_band(int img_height, int img_width, int row_begin, int row_end, int channels, int num_points,
                                   const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                                   const float *colors, const float *v_output_band, const uint16_t *tile_topk, float *v_xy, float *v_conic,
                                   float *v_colors, void *stream) {
    IGS_REQUIRE(tile_topk != nullptr, "igs_raster_bwd_topk_tiles_band: null tile_topk");
    IGS_REQUIRE(row_end >= 0, "igs_raster_bwd_topk_tiles_band: negative row_end");
    return raster_bwd(img_height, img_width, row_begin, row_end, channels, num_points, gaussian_ids_sorted, tile_bins, xys, conics, colors,
                      v_output_band, nullptr, tile_topk, v_xy, v_conic, v_colors, stream, "igs_raster_bwd_topk_tiles_band");
}

int igs_raster_step_l1_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                            int num_points, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                            const float *conics, const float *colors, const float *target, float ratio, float *out_img, float *loss,
                            float *v_output, float *v_xy, float *v_conic, float *v_colors, void *workspace, size_t workspace_bytes,
                            void *stream) {
    return raster_step(tiles_x, tiles_y, img_height, img_width, row_begin, row_end, channels, num_points, gaussian_ids_sorted, tile_bins,
                       xys, conics, colors, target, ratio, out_img, loss, v_output, v_xy, v_conic, v_colors, workspace, workspace_bytes,
                       stream, "igs_raster_step_l1_band");
}

int igs_raster_step_l1(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int num_points,
                       const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                       const float *colors, const float *target, float ratio, float *out_img, float *loss, float *v_output, float *v_xy,
                       float *v_conic, float *v_colors, void *workspace, size_t workspace_bytes, void *stream) {
    return raster_step(tiles_x, tiles_y, img_height, img_width, 0, tiles_y, channels, num_points, gaussian_ids_sorted, tile_bins, xys,
                       conics, colors, target, ratio, out_img, loss, v_output, v_xy, v_conic, v_colors, workspace, workspace_bytes, stream,
                       "igs_raster_step_l1");
}

}  // extern "C"

namespace igs {

int raster_step_fused(int tiles_x, int tiles_y, int img_h, int img_w, int row_begin, int row_end, int channels, int num_points,
                      const int32_t *ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics, const float *colors,
                      const float *target, float ratio, float *out_img, float *loss, float *v_xy, float *v_conic, float *v_colors,
                      void *workspace, size_t workspace_bytes, bool finish_loss, cudaStream_t s) {
    return raster_step(tiles_x, tiles_y, img_h, img_w, row_begin, row_end, channels, num_points, ids_sorted, tile_bins, xys, conics, colors,
                       target, ratio, out_img, loss, nullptr, v_xy, v_conic, v_colors, workspace, workspace_bytes, s, "raster (training step)",
                       true, finish_loss);
}

}  // namespace igs

