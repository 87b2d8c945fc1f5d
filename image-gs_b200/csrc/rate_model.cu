// Fixed inputs of the rate term (compress/rate.py:131-164, rate_model; with predicting_sources 116-128 and channel_operands 69-78), built
// on the GPU from the quantized Gaussians once their neighbours are known (igs_nearest_neighbors in bitstream order):
//   * per Gaussian: the neighbours clamped to valid indices, their weights 1 / count (0 for missing ones), the CCLM slope of each channel
//     (covariance over variance plus the squared step of the reference channel's neighbour values, clamped to +-4, only for channels with
//     a prediction reference and Gaussians with at least 3 neighbours), and the residual of its prediction in quantization steps, rounded;
//   * per channel: 1 / (scale ln 2) of the Laplace distribution whose scale is the mean absolute rounded residual (at least 0.3);
//   * per Gaussian: 1 / (scale ln 2) of its rotation's distribution, the scale being the mean absolute rotation index of its aspect-ratio
//     class (classes by |log2 s0 - log2 s1| against 0.25, 0.5, 1 and 2 octaves; an empty class takes the mean over all, at least 0.3);
//   * the Gaussians that predict from each Gaussian (CSR lists in increasing order) and their weights of it.
// Float operations follow the reference's float32 order one rounding at a time (__fmul_rn / __fadd_rn / __fdiv_rn: no contraction); the
// two means are of integers (rounded residuals, rotation indices) and are summed exactly in 64-bit integers, then divided as the
// reference's float32 mean does. IEEE build (no fast-math).
#include <climits>

#include "igs_common.cuh"
#include "radix_sort.cuh"

namespace {

using igs::kMaxChannels;
constexpr int kThreads = 256;
constexpr int kNeighbors = 8;       // NUM_NEIGHBORS of compress/prediction.py
constexpr int kClasses = 5;         // aspect-ratio classes: boundaries 0.25, 0.5, 1, 2 octaves
constexpr float kMinScale = 0.3f;   // MIN_SCALE
constexpr float kMaxSlope = 4.0f;   // MAX_SLOPE
constexpr int kMinCclm = 3;         // MIN_CCLM_NEIGHBORS
constexpr float kLn2 = 0.693147182f;  // float32 of ln 2, as a float32 tensor times math.log(2.0)

struct Refs {
    int color[kMaxChannels];  // channel subtracted before the prediction, -1 for none
    int pred[kMaxChannels];   // prediction reference channel, -1 for none
};

struct Accumulators {
    unsigned long long abs_residual[kMaxChannels];  // sums of |rounded residual| per channel
    unsigned long long class_rot[kClasses];         // sums of |rotation index| per class
    unsigned long long class_count[kClasses];
    unsigned long long all_rot;                     // sum of |rotation index| over all Gaussians
    float class_inv[kClasses];                      // 1 / (class scale ln 2)
};

__device__ __forceinline__ int aspect_class(float ls0, float ls1) {
    const float d = fabsf(__fsub_rn(ls0, ls1));
    // torch.bucketize(right=False): the number of boundaries strictly below d
    return (d > 0.25f) + (d > 0.5f) + (d > 1.0f) + (d > 2.0f);
}

// the feature values after the colour-reference subtraction (coded_values): f_c - f_ref * [ref >= 0]
template <int kMaxC>
__device__ __forceinline__ void coded_values(const float *__restrict__ f, const Refs &refs, int channels, float (&v)[kMaxC]) {
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        v[c] = 0.f;
        if (c >= channels) continue;
        const int r = refs.color[c];
        v[c] = __fsub_rn(f[c], r >= 0 ? __fmul_rn(f[r], 1.f) : __fmul_rn(f[c], 0.f));
    }
}

template <int C>
__global__ void __launch_bounds__(kThreads) gaussian_kernel(const int n, const int channels_rt, const Refs refs,
                                                            const long long *__restrict__ neighbors, const float *__restrict__ feat,
                                                            const float *__restrict__ log2_scale, const float *__restrict__ q_rot,
                                                            const float *__restrict__ steps, int *__restrict__ neighbors_out,
                                                            float *__restrict__ weights, float *__restrict__ slope,
                                                            int *__restrict__ in_degree, unsigned char *__restrict__ count_out,
                                                            unsigned char *__restrict__ class_out, Accumulators *__restrict__ acc) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    // the block's integer sums in shared memory, added to the global ones once per block
    __shared__ unsigned long long s_abs[kMaxChannels], s_rot[kClasses], s_cnt[kClasses], s_all;
    if (threadIdx.x < kMaxChannels) s_abs[threadIdx.x] = 0ull;
    if (threadIdx.x < kClasses) s_rot[threadIdx.x] = 0ull, s_cnt[threadIdx.x] = 0ull;
    if (threadIdx.x == 0) s_all = 0ull;
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        int nb[kNeighbors];
        float valid[kNeighbors], w[kNeighbors];
        int count = 0;
#pragma unroll
        for (int k = 0; k < kNeighbors; ++k) {
            const long long j = neighbors[(size_t)i * kNeighbors + k];
            const bool ok = j >= 0 && j < n;
            nb[k] = ok ? (int)j : 0;
            valid[k] = ok ? 1.f : 0.f;
            count += ok;
            if (ok) atomicAdd(&in_degree[j], 1);
        }
        const float countf = (float)count;
#pragma unroll
        for (int k = 0; k < kNeighbors; ++k) {
            w[k] = __fdiv_rn(valid[k], fmaxf(countf, 1.f));
            neighbors_out[(size_t)i * kNeighbors + k] = nb[k];
            weights[(size_t)i * kNeighbors + k] = w[k];
        }
        count_out[i] = (unsigned char)count;

        // neighbour means, covariances with the reference channel, and variances (sums over the neighbours in order)
        float mean[kMaxC], cov[kMaxC], var[kMaxC];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) mean[c] = 0.f, cov[c] = 0.f, var[c] = 0.f;
#pragma unroll
        for (int k = 0; k < kNeighbors; ++k) {
            float v[kMaxC];
            coded_values<kMaxC>(feat + (size_t)nb[k] * channels, refs, channels, v);
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) {
                if (c >= channels) continue;
                const int p = refs.pred[c] >= 0 ? refs.pred[c] : c;
                const float nv = __fmul_rn(v[c], valid[k]), np = __fmul_rn(v[p], valid[k]);
                mean[c] = __fadd_rn(mean[c], __fmul_rn(nv, w[k]));
                cov[c] = __fadd_rn(cov[c], __fmul_rn(__fmul_rn(nv, np), w[k]));
                var[c] = __fadd_rn(var[c], __fmul_rn(__fmul_rn(np, np), w[k]));
            }
        }
        float own[kMaxC], s[kMaxC];
        coded_values<kMaxC>(feat + (size_t)i * channels, refs, channels, own);
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            s[c] = 0.f;
            if (c >= channels) continue;
            const int p = refs.pred[c] >= 0 ? refs.pred[c] : c;
            const float cv = __fsub_rn(cov[c], __fmul_rn(mean[c], mean[p]));
            const float vr = __fsub_rn(var[c], __fmul_rn(mean[p], mean[p]));
            const float ratio = __fdiv_rn(cv, __fadd_rn(vr, __fmul_rn(steps[c], steps[c])));
            const float clamped = fminf(fmaxf(ratio, -kMaxSlope), kMaxSlope);
            s[c] = __fmul_rn(__fmul_rn(clamped, refs.pred[c] >= 0 ? 1.f : 0.f), count >= kMinCclm ? 1.f : 0.f);
            slope[(size_t)i * channels + c] = s[c];
        }
        // the rounded residual of the prediction in steps (feature_residuals): (v - m - slope (v_ref - m_ref)) / step, half to even
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            if (c >= channels) continue;
            const int p = refs.pred[c] >= 0 ? refs.pred[c] : c;
            const float dev = __fsub_rn(own[p], mean[p]);
            const float r = __fmul_rn(__fsub_rn(__fsub_rn(own[c], mean[c]), __fmul_rn(s[c], dev)), __fdiv_rn(1.f, steps[c]));
            atomicAdd(&s_abs[c], (unsigned long long)fabsf(rintf(r)));
        }
        // rotation statistics of the aspect-ratio class
        const int cls = aspect_class(log2_scale[2 * (size_t)i], log2_scale[2 * (size_t)i + 1]);
        class_out[i] = (unsigned char)cls;
        const unsigned long long a = (unsigned long long)fabsf(q_rot[i]);
        atomicAdd(&s_rot[cls], a);
        atomicAdd(&s_cnt[cls], 1ull);
        atomicAdd(&s_all, a);
    }
    __syncthreads();
    if (threadIdx.x < channels) atomicAdd(&acc->abs_residual[threadIdx.x], s_abs[threadIdx.x]);
    if (threadIdx.x < kClasses) {
        atomicAdd(&acc->class_rot[threadIdx.x], s_rot[threadIdx.x]);
        atomicAdd(&acc->class_count[threadIdx.x], s_cnt[threadIdx.x]);
    }
    if (threadIdx.x == 0) atomicAdd(&acc->all_rot, s_all);
}

// one thread: the per-channel scales and coefficients and the per-class rotation coefficients
__global__ void scalars_kernel(const int n, const int channels, const float *__restrict__ steps, const float *__restrict__ channel_weights,
                               float *__restrict__ inv_steps, float *__restrict__ inv_feat, float *__restrict__ feat_coeffs,
                               Accumulators *__restrict__ acc) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const float nf = (float)n;
    for (int c = 0; c < channels; ++c) {
        inv_steps[c] = __fdiv_rn(1.f, steps[c]);
        const float mean_abs = __fdiv_rn((float)acc->abs_residual[c], nf);
        const float inv = __fdiv_rn(1.f, __fmul_rn(fmaxf(mean_abs, kMinScale), kLn2));
        inv_feat[c] = inv;
        feat_coeffs[c] = __fmul_rn(inv, channel_weights[c]);
    }
    const float all_mean = __fdiv_rn((float)acc->all_rot, nf);
    for (int k = 0; k < kClasses; ++k) {
        const float cnt = (float)acc->class_count[k];
        const float scale = acc->class_count[k] > 0 ? __fdiv_rn((float)acc->class_rot[k], fmaxf(cnt, 1.f)) : all_mean;
        acc->class_inv[k] = __fdiv_rn(1.f, __fmul_rn(fmaxf(scale, kMinScale), kLn2));
    }
}

__global__ void __launch_bounds__(kThreads) rot_kernel(const int n, const unsigned char *__restrict__ class_of,
                                                       const Accumulators *__restrict__ acc, float *__restrict__ inv_rot) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) inv_rot[i] = acc->class_inv[class_of[i]];
}

// The in-neighbour lists (compress/rate.py:116-128, predicting_sources: the rows of the neighbour matrix stably sorted by target): every
// (Gaussian i, neighbour slot k) entry in row-major order keyed by its neighbour j (invalid ones by num_points, after all valid ones), for
// a stable radix sort by key, which leaves each list in increasing i without a per-list sort (whose cost grows with the square of a
// list's length, and one Gaussian can be a neighbour of thousands)
__global__ void __launch_bounds__(kThreads) source_keys_kernel(const int n, const long long *__restrict__ neighbors,
                                                               unsigned long long *__restrict__ keys, int *__restrict__ values) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * kNeighbors) return;
    const long long j = neighbors[t];
    keys[t] = (j < 0 || j >= n) ? (unsigned long long)n : (unsigned long long)j;
    values[t] = t / kNeighbors;
}

// the sorted entries' Gaussians and their weights, 1 / their neighbour counts: the first offsets[n] entries are the valid ones
__global__ void __launch_bounds__(kThreads) sources_kernel(const int n, const int *__restrict__ offsets, const int *__restrict__ sorted,
                                                           const unsigned char *__restrict__ counts, int *__restrict__ sources,
                                                           float *__restrict__ source_weights) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= offsets[n]) return;
    const int i = sorted[t];
    sources[t] = i;
    source_weights[t] = __fdiv_rn(1.f, (float)counts[i]);
}

size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

struct Layout {
    size_t acc, in_degree, counts, classes, keys0, keys1, vals0, vals1, radix_counts, cum, total;
};

Layout layout(int n) {
    const size_t entries = (size_t)n * kNeighbors;
    Layout l;
    size_t off = 0;
    l.acc = off, off += round256(sizeof(Accumulators));
    l.in_degree = off, off += round256(sizeof(int) * (size_t)n);
    l.counts = off, off += round256((size_t)n);
    l.classes = off, off += round256((size_t)n);
    l.keys0 = off, off += round256(sizeof(unsigned long long) * entries);
    l.keys1 = off, off += round256(sizeof(unsigned long long) * entries);
    l.vals0 = off, off += round256(sizeof(int) * entries);
    l.vals1 = off, off += round256(sizeof(int) * entries);
    l.radix_counts = off, off += round256(radix::counts_bytes((int)entries));
    l.cum = off, off += round256(igs_cumsum_workspace(n));
    l.total = off;
    return l;
}

}  // namespace

extern "C" {

size_t igs_rate_model_workspace(int num_points) { return layout(num_points > 0 ? num_points : 1).total; }

int igs_rate_model(int num_points, int channels, const int64_t *neighbors, const float *feat, const float *log2_scale, const float *q_rot,
                   const int32_t *color_refs, const int32_t *pred_refs, const float *steps, const float *channel_weights,
                   int32_t *neighbors_out, float *weights, float *slope, float *inv_steps, float *inv_feat, float *feat_coeffs,
                   float *inv_rot, int32_t *offsets, int32_t *sources, float *source_weights, void *workspace, size_t workspace_bytes,
                   void *stream) {
    const char *who = "igs_rate_model";
    IGS_REQUIRE(num_points >= 0 && num_points <= INT_MAX / kNeighbors, "%s: %d Gaussians (at most %d)", who, num_points,
                INT_MAX / kNeighbors);
    IGS_REQUIRE(channels >= 1 && channels <= kMaxChannels, "%s: 1 to %d channels (got %d)", who, kMaxChannels, channels);
    IGS_REQUIRE(color_refs && pred_refs, "%s: null channel references", who);
    Refs refs;
    for (int c = 0; c < kMaxChannels; ++c) refs.color[c] = refs.pred[c] = -1;
    for (int c = 0; c < channels; ++c) {
        IGS_REQUIRE(color_refs[c] >= -1 && color_refs[c] < channels && color_refs[c] != c, "%s: bad colour reference %d of channel %d",
                    who, color_refs[c], c);
        IGS_REQUIRE(pred_refs[c] >= -1 && pred_refs[c] < channels && pred_refs[c] != c, "%s: bad prediction reference %d of channel %d",
                    who, pred_refs[c], c);
        refs.color[c] = color_refs[c];
        refs.pred[c] = pred_refs[c];
    }
    IGS_REQUIRE(steps && channel_weights && inv_steps && inv_feat && feat_coeffs && offsets && workspace, "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || (neighbors && feat && log2_scale && q_rot && neighbors_out && weights && slope && inv_rot && sources &&
                                    source_weights),
                "%s: null pointer", who);
    const Layout l = layout(num_points > 0 ? num_points : 1);
    IGS_REQUIRE(workspace_bytes >= l.total, "%s: workspace too small (%zu bytes, need %zu)", who, workspace_bytes, l.total);
    IGS_REQUIRE(igs::aligned(workspace, 16), "%s: workspace must be 16-byte aligned", who);
    cudaStream_t s = igs::as_stream(stream);
    char *ws = static_cast<char *>(workspace);
    Accumulators *acc = reinterpret_cast<Accumulators *>(ws + l.acc);
    int *in_degree = reinterpret_cast<int *>(ws + l.in_degree);
    unsigned char *counts = reinterpret_cast<unsigned char *>(ws + l.counts);
    unsigned char *classes = reinterpret_cast<unsigned char *>(ws + l.classes);
    unsigned long long *keys[2] = {reinterpret_cast<unsigned long long *>(ws + l.keys0), reinterpret_cast<unsigned long long *>(ws + l.keys1)};
    int *vals[2] = {reinterpret_cast<int *>(ws + l.vals0), reinterpret_cast<int *>(ws + l.vals1)};
    // accumulators and in-degrees start at zero (one memset: they are the first bytes of the workspace)
    if (cudaMemsetAsync(ws, 0, l.counts, s) != cudaSuccess) return igs::check_launch(who);  // acc and in_degree
    if (cudaMemsetAsync(offsets, 0, sizeof(int32_t), s) != cudaSuccess) return igs::check_launch(who);
    const int blocks = igs::ceil_div(num_points > 0 ? num_points : 1, kThreads);
    if (num_points > 0) {
        const auto kernel = channels == 3 ? gaussian_kernel<3> : gaussian_kernel<0>;
        kernel<<<blocks, kThreads, 0, s>>>(num_points, channels, refs, reinterpret_cast<const long long *>(neighbors), feat, log2_scale,
                                           q_rot, steps, neighbors_out, weights, slope, in_degree, counts, classes, acc);
        const int status = igs_cumsum(num_points, in_degree, offsets + 1, nullptr, ws + l.cum, l.total - l.cum, stream);
        if (status != IGS_OK) return status;
    }
    scalars_kernel<<<1, 32, 0, s>>>(num_points, channels, steps, channel_weights, inv_steps, inv_feat, feat_coeffs, acc);
    if (num_points > 0) {
        rot_kernel<<<blocks, kThreads, 0, s>>>(num_points, classes, acc, inv_rot);
        const int entries = num_points * kNeighbors;
        const int entry_blocks = igs::ceil_div(entries, kThreads);
        source_keys_kernel<<<entry_blocks, kThreads, 0, s>>>(num_points, reinterpret_cast<const long long *>(neighbors), keys[0], vals[0]);
        const int cur = radix::sort_pairs(entries, radix::bit_length((unsigned long long)num_points),
                                          keys, vals, reinterpret_cast<int *>(ws + l.radix_counts), s);
        sources_kernel<<<entry_blocks, kThreads, 0, s>>>(num_points, offsets, vals[cur], counts, sources, source_weights);
    }
    return igs::check_launch(who);
}

}  // extern "C"
