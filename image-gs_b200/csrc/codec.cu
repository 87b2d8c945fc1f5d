// Entropy coding of the bitstream's integer streams (compress/rans_codec.py over compress/csrc/rans.cpp): each stream of one value per
// Gaussian is coded as its raw values or as differences between consecutive ones, mapped to non-negative integers by a shift to its
// minimum or a zigzag around its rounded median, split into tokens and raw low bits (values below 2^split_exp are their own token, larger
// ones their bit length and msb_bits leading bits, the rest raw), with a static token histogram of log-quantized counts; every stream
// shares one 64-bit rANS state (32-bit renormalisation, frequencies summing to 2^16, raw bits as uniform symbols of at most 16 bits).
//
// The encoder picks, per stream, the mapping and the token model of the smallest estimated size among the same candidates, in the same
// order and with the same double-precision arithmetic as the reference (its costs are sums in numpy's pairwise order), so both write the
// same bytes. The model search reads only each candidate's histogram of fine tokens; the candidates (raw or differences, shift or
// zigzag) are fitted on host threads. Decoding is one serial pass over the rANS state.
//
// The estimate of a stream's coded size used for rate decisions during training (estimate_stream_bits) takes device streams: its
// histograms of fine tokens are built on the GPU (one launch for every stream and both mappings), the formula on the host.
//
// Everything here is host code except the histogram kernels; the data are small (one value per Gaussian and attribute channel) and the
// coder is serial, so the GPU is used where a pass over the values is parallel.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <exception>
#include <memory>
#include <thread>
#include <vector>

#include "igs_common.cuh"

namespace {

constexpr int kPrec = 16;                   // token frequencies sum to 2^kPrec
constexpr int kRawChunk = 16;               // raw bits per uniform symbol, at most
constexpr uint64_t kStateLow = 1ull << 31;  // lower bound of the rANS state
constexpr int kMaxSplitExp = 12;
constexpr int kMaxMsbBits = 3;
constexpr int kMaxMantissaBits = 3;
constexpr int kEstimateTableBits = 6;  // estimated header bits per used token of estimate_stream_bits
constexpr int kMaxExponent = 62;       // of values and count weights (int64)
constexpr int kMaxTokens = IGS_RANS_MAX_TOKENS;
static_assert((1 << kMaxSplitExp) + ((kMaxExponent - kMaxSplitExp + 1) << kMaxMsbBits) <= kMaxTokens, "token space");

using I64 = std::vector<int64_t>;

__host__ __device__ inline int bits_of(int64_t v) {  // bit length of a non-negative integer
#ifdef __CUDA_ARCH__
    return v == 0 ? 0 : 64 - __clzll(v);
#else
    return v == 0 ? 0 : 64 - __builtin_clzll((unsigned long long)v);
#endif
}

inline int64_t exp_golomb_bits(int64_t v) { return 2 * bits_of(v + 1) - 1; }

__host__ __device__ inline int64_t zigzag(int64_t v) { return (int64_t)(((uint64_t)v << 1) ^ (uint64_t)(v >> 63)); }

// token of a non-negative value, its raw low bits and their number
struct Split {
    int64_t token, raw;
    int num_raw;
};

__host__ __device__ inline Split split_value(int64_t v, int split_exp, int msb_bits) {
    const int64_t first = int64_t(1) << split_exp;
    if (v < first) return {v, 0, 0};
    const int top = bits_of(v) - 1;
    const int num_raw = top - msb_bits;
    const int64_t lead = (v >> num_raw) & ((int64_t(1) << msb_bits) - 1);
    return {first + (int64_t(top - split_exp) << msb_bits) + lead, v & ((int64_t(1) << num_raw) - 1), num_raw};
}

// the smallest value of a token and its number of raw bits
inline void token_base(int64_t token, int split_exp, int msb_bits, int64_t &base, int &num_raw) {
    const int64_t first = int64_t(1) << split_exp;
    if (token < first) {
        base = token, num_raw = 0;
        return;
    }
    num_raw = split_exp + (int)((token - first) >> msb_bits) - msb_bits;
    base = ((int64_t(1) << msb_bits) | ((token - first) & ((int64_t(1) << msb_bits) - 1))) << num_raw;
}

// log-quantized count code (0 for unused tokens) and the weight it stands for
inline int64_t count_code(int64_t count, int mantissa_bits) {
    if (count < (int64_t(2) << mantissa_bits)) return count;
    int e = std::max(bits_of(count) - (mantissa_bits + 1), 0);
    int64_t m = (count + (e > 0 ? int64_t(1) << std::max(e - 1, 0) : 0)) >> e;
    if (m == (int64_t(2) << mantissa_bits)) m = int64_t(1) << mantissa_bits, ++e;
    return (int64_t(e) << mantissa_bits) + m;
}

inline bool code_to_weight(int64_t code, int mantissa_bits, int64_t &weight) {
    if (code < (int64_t(2) << mantissa_bits)) {
        weight = code;
        return code >= 0;
    }
    const int64_t e = (code >> mantissa_bits) - 1;
    if (e > kMaxExponent - kPrec - (mantissa_bits + 1)) return false;
    weight = (code - (e << mantissa_bits)) << e;
    return true;
}

// frequencies summing to 2^kPrec, at least 1 for every token of positive weight; the rest goes to the first largest
inline bool frequencies(const I64 &weights, I64 &freqs) {
    int64_t total = 0;
    for (int64_t w : weights) total += w;
    if (total <= 0) return false;
    freqs.assign(weights.size(), 0);
    int64_t sum = 0;
    size_t top = 0;
    for (size_t i = 0; i < weights.size(); ++i) {
        freqs[i] = weights[i] > 0 ? std::max<int64_t>((weights[i] << kPrec) / total, 1) : 0;
        sum += freqs[i];
        if (freqs[i] > freqs[top]) top = i;
    }
    freqs[top] += (int64_t(1) << kPrec) - sum;
    return freqs[top] >= 1;
}

// header bits of a table of count codes after its length and mantissa bits: a flag, then fixed-width or Exp-Golomb-coded differences
inline int64_t table_cost(const I64 &codes) {
    const int64_t fixed = 5 + (int64_t)codes.size() * bits_of(*std::max_element(codes.begin(), codes.end()));
    int64_t delta = 0, prev = 0;
    for (int64_t c : codes) delta += exp_golomb_bits(zigzag(c - prev)), prev = c;
    return 1 + std::min(fixed, delta);
}

// kPrec - log2(f) for every frequency f
const std::vector<double> &symbol_bits() {
    static const std::vector<double> table = [] {
        std::vector<double> t((size_t(1) << kPrec) + 1, 0.0);
        for (size_t f = 1; f < t.size(); ++f) t[f] = kPrec - std::log2((double)f);
        return t;
    }();
    return table;
}

// the sum of the values in the order of numpy's pairwise summation (blocks of 8 partial sums below 128 values, halves above), which the
// reference's costs follow, so that equal costs compare equal
double numpy_sum(const double *v, size_t n) {
    if (n < 8) {
        double s = 0.0;
        for (size_t i = 0; i < n; ++i) s += v[i];
        return s;
    }
    if (n <= 128) {
        double r[8];
        for (int j = 0; j < 8; ++j) r[j] = v[j];
        size_t i = 8;
        for (; i < n - n % 8; i += 8)
            for (int j = 0; j < 8; ++j) r[j] += v[i + j];
        double s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; ++i) s += v[i];
        return s;
    }
    size_t half = n / 2;
    half -= half % 8;
    return numpy_sum(v, half) + numpy_sum(v + half, n - half);
}

// the non-empty tokens of a fine histogram as (smallest value, count), in increasing order
struct FineBin {
    int64_t base, count;
};

std::vector<FineBin> fine_bins(const I64 &fine, int fine_split, int fine_msb) {
    std::vector<FineBin> bins;
    for (size_t t = 0; t < fine.size(); ++t) {
        if (fine[t] == 0) continue;
        int64_t base;
        int nr;
        token_base((int64_t)t, fine_split, fine_msb, base, nr);
        bins.push_back({base, fine[t]});
    }
    return bins;
}

// the histogram of a coarser tokenizer (split_exp <= fine_split, msb_bits <= fine_msb) from a fine one: every value of a fine token has
// the same coarse token and raw-bit count, those of the fine token's smallest value, and coarse tokens increase with the value, so the
// last bin gives the histogram's length. Returns the raw bits.
int64_t coarsen(const std::vector<FineBin> &bins, int split_exp, int msb_bits, I64 &counts) {
    counts.assign(bins.empty() ? 0 : (size_t)split_value(bins.back().base, split_exp, msb_bits).token + 1, 0);
    int64_t raw_bits = 0;
    for (const FineBin &b : bins) {
        const Split sp = split_value(b.base, split_exp, msb_bits);
        counts[sp.token] += b.count;
        raw_bits += b.count * sp.num_raw;
    }
    return raw_bits;
}

struct TokenModel {
    int split_exp = 0, msb_bits = 0, mantissa_bits = 0;
    I64 codes, freqs;
    double payload_bits = 0.0, bits = 0.0;
};

// the fine tokenizer of a stream whose largest mapped value is vmax
inline void fine_tokenizer(int64_t vmax, int &split, int &msb) {
    split = std::min(bits_of(vmax), kMaxSplitExp);
    msb = std::min(split, kMaxMsbBits);
}

// The token model of the smallest estimated size for a stream of n values with the given fine histogram: every tokenizer (split_exp,
// msb_bits) and count quantization (mantissa_bits) in increasing order, the first of equal sizes kept; a tokenizer whose lower bound
// (the entropy of its token counts plus the smallest header) cannot beat the best so far is skipped, as the reference does.
TokenModel best_model(const I64 &fine, int fine_split, int fine_msb, int64_t n) {
    const std::vector<double> &len = symbol_bits();
    const std::vector<FineBin> bins = fine_bins(fine, fine_split, fine_msb);
    TokenModel best;
    bool have = false;
    I64 counts, codes, weights, freqs;
    std::vector<double> terms;
    for (int split = 0; split <= fine_split; ++split) {
        for (int msb = 0; msb <= std::min(split, kMaxMsbBits); ++msb) {
            const int64_t raw_bits = coarsen(bins, split, msb, counts);
            const int64_t header = 4 + 2 + exp_golomb_bits((int64_t)counts.size() - 1) + 2;
            if (have) {
                terms.clear();
                for (int64_t c : counts)
                    if (c > 0) terms.push_back((double)c * std::log2((double)n / (double)c));
                const double bound = (double)(header + 1 + (int64_t)counts.size()) + numpy_sum(terms.data(), terms.size()) + (double)raw_bits;
                if (bound > best.bits * (1.0 + 1e-9) + 1e-6) continue;
            }
            codes.resize(counts.size());
            weights.resize(counts.size());
            for (int mb = 0; mb <= kMaxMantissaBits; ++mb) {
                for (size_t t = 0; t < counts.size(); ++t) {
                    codes[t] = count_code(counts[t], mb);
                    code_to_weight(codes[t], mb, weights[t]);
                }
                frequencies(weights, freqs);
                terms.clear();
                for (size_t t = 0; t < counts.size(); ++t)
                    if (counts[t] > 0) terms.push_back((double)counts[t] * len[freqs[t]]);
                const double payload = numpy_sum(terms.data(), terms.size());
                const double bits = (double)(header + table_cost(codes)) + payload + (double)raw_bits;
                if (!have || bits < best.bits) {
                    have = true;
                    best.split_exp = split, best.msb_bits = msb, best.mantissa_bits = mb;
                    best.codes = codes, best.freqs = freqs;
                    best.payload_bits = payload + (double)raw_bits;
                    best.bits = bits;
                }
            }
        }
    }
    return best;
}

// int(np.round(np.median(values))) of the n values value(0) ... value(n - 1), all in [lo, hi]: the middle value, or the mean of the two
// middle ones, rounded half to even. Exact selection in two passes: a histogram of the values' offsets from lo in at most 2^12 buckets
// finds the buckets of the middle ranks, and only the values in those buckets are ordered.
template <typename Value>
int64_t median_rounded(size_t n, Value value, int64_t lo, int64_t hi) {
    const size_t half = n / 2;
    const uint64_t range = (uint64_t)hi - (uint64_t)lo;
    const int width = range == 0 ? 0 : 64 - __builtin_clzll(range);
    const int shift = std::max(0, width - 12);
    std::vector<uint32_t> hist((size_t)(range >> shift) + 1, 0u);
    for (size_t i = 0; i < n; ++i) ++hist[((uint64_t)value(i) - (uint64_t)lo) >> shift];
    const size_t first_rank = n % 2 ? half : half - 1;  // the lower middle rank (the only one for odd n)
    size_t below = 0, b_lo = 0;
    while (below + hist[b_lo] <= first_rank) below += hist[b_lo++];
    size_t b_hi = b_lo, below_hi = below;
    while (below_hi + hist[b_hi] <= half) below_hi += hist[b_hi++];
    I64 mid;
    mid.reserve(below_hi + hist[b_hi] - below);
    for (size_t i = 0; i < n; ++i) {
        const int64_t x = value(i);
        const size_t b = (size_t)(((uint64_t)x - (uint64_t)lo) >> shift);
        if (b >= b_lo && b <= b_hi) mid.push_back(x);
    }
    std::nth_element(mid.begin(), mid.begin() + (half - below), mid.end());  // mid[i] holds the value of rank below + i
    double m = (double)mid[half - below];
    if (n % 2 == 0) m = ((double)*std::max_element(mid.begin(), mid.begin() + (half - below)) + m) / 2.0;
    return (int64_t)std::nearbyint(m);
}

struct Fit {
    double bits = 0.0;
    bool delta = false, zigzag_mapped = false;
    int64_t param = 0;
    TokenModel model;
};

// The value of index i of a stream as coded: its raw value or its difference with the previous one, shifted or zigzagged around param
struct Mapping {
    const int64_t *v;
    bool delta, zz;
    int64_t param;
    int64_t candidate(size_t i) const { return delta ? v[i] - (i > 0 ? v[i - 1] : 0) : v[i]; }
    int64_t operator()(size_t i) const { return zz ? zigzag(candidate(i) - param) : candidate(i) - param; }
};

// One mapping of a stream's raw values (delta = false) or differences between consecutive values (delta = true) to non-negative
// integers, a shift to the minimum (zz = false) or a zigzag around the rounded median (zz = true), with its best token model. The
// encoder keeps, per stream, the first of the smallest size in the order (raw, shift), (raw, zigzag), (differences, shift),
// (differences, zigzag), as the reference does. The mapped values are not stored: the rANS pass maps them again.
Fit fit_one(const int64_t *v, size_t n, bool delta, bool zz) {
    Mapping map{v, delta, zz, 0};
    int64_t lo = map.candidate(0), hi = lo;
    for (size_t i = 1; i < n; ++i) {
        const int64_t x = map.candidate(i);
        lo = std::min(lo, x), hi = std::max(hi, x);
    }
    map.param = zz ? median_rounded(n, [&](size_t i) { return map.candidate(i); }, lo, hi) : lo;
    // the largest mapped value: zigzag grows with the distance from param on either side
    const int64_t vmax = zz ? std::max(zigzag(hi - map.param), zigzag(lo - map.param)) : hi - lo;
    int split, msb;
    fine_tokenizer(vmax, split, msb);
    I64 fine(split_value(vmax, split, msb).token + 1, 0);  // tokens increase with the value
    for (size_t i = 0; i < n; ++i) ++fine[split_value(map(i), split, msb).token];
    Fit f;
    f.delta = delta, f.zigzag_mapped = zz, f.param = map.param;
    f.model = best_model(fine, split, msb, (int64_t)n);
    f.bits = (double)(1 + exp_golomb_bits(zigzag(f.param))) + f.model.bits;
    return f;
}

// fn(0) ... fn(n - 1) on up to num_threads host threads (0: one per hardware thread), the calling thread included
template <typename Fn>
void parallel_for(size_t n, Fn fn, int num_threads = 0) {
    std::atomic<size_t> next{0};
    auto work = [&]() {
        for (size_t t = next++; t < n; t = next++) fn(t);
    };
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>(n, num_threads > 0 ? (size_t)num_threads : hw);
    std::vector<std::thread> pool;
    for (size_t t = 1; t < threads; ++t) pool.emplace_back(work);
    work();
    for (std::thread &t : pool) t.join();
}

// One token of a stream's model as the encoder uses it: x / freq for 0 <= x < 2^63 and 1 <= freq <= 2^16 by a multiply-high and a
// shift (Granlund and Montgomery, "Division by Invariant Integers using Multiplication", 1994, theorem 4.2 with N = 63: with
// l = ceil(log2 freq) and m = ceil(2^(63 + l) / freq), which is below 2^64, floor(x / freq) = floor(m x / 2^(63 + l)), taken as the
// high word of (2 x) m shifted right by l); the state before a token is below x_max <= 2^63. The update ((x / freq) << kPrec) +
// x % freq + start is x + start + q (2^kPrec - freq).
struct EncToken {
    uint64_t x_max, rcp;
    uint32_t start, cmpl;
    int shift;
};

std::vector<EncToken> encoder_tokens(const I64 &freqs) {
    std::vector<EncToken> tokens(freqs.size());
    int64_t start = 0;
    for (size_t t = 0; t < freqs.size(); ++t) {
        const uint64_t f = (uint64_t)freqs[t];
        EncToken &e = tokens[t];
        e.start = (uint32_t)start, e.cmpl = (uint32_t)((uint64_t(1) << kPrec) - f);
        start += freqs[t];
        if (f == 0) continue;  // an unused token
        e.x_max = ((kStateLow >> kPrec) << 32) * f;
        const int l = f == 1 ? 0 : 64 - __builtin_clzll(f - 1);
        e.shift = l;
        const unsigned __int128 num = (unsigned __int128)1 << (63 + l);
        e.rcp = (uint64_t)((num + f - 1) / f);
    }
    return tokens;
}

// The rANS state over every stream's symbols, encoded last to first (the decoder reads stream 0's first value first: its token, then
// its raw bits in chunks of at most kRawChunk bits, most significant first, each a uniform symbol of that many bits). The 32-bit words
// the state emits are written backward from the end of words[0, capacity); the payload is the final state's high and low words followed
// by the emitted words, last emitted first. Returns the index of the payload's first word, or -1 when it does not fit.
int64_t rans_pack(const std::vector<Mapping> &mapped, size_t n, const std::vector<std::vector<EncToken>> &tokens, const int *split_exp,
                  const int *msb_bits, uint32_t *words, int64_t capacity) {
    constexpr int kMaxWordsPerValue = 1 + (kMaxExponent + kRawChunk - 1) / kRawChunk;
    uint64_t x = kStateLow;
    int64_t pos = capacity;
    // emit the low word when x >= limit: the word is stored either way (a later one overwrites it when not emitted), no branch
    auto renorm = [&](uint64_t limit) {
        words[pos - 1] = (uint32_t)x;
        const bool out = x >= limit;
        pos -= out;
        x = out ? x >> 32 : x;
    };
    for (size_t s = mapped.size(); s-- > 0;) {
        const EncToken *tok = tokens[s].data();
        const Mapping &map = mapped[s];
        const int split = split_exp[s], msb = msb_bits[s];
        for (size_t i = n; i-- > 0;) {
            if (pos < kMaxWordsPerValue) return -1;
            const Split sp = split_value(map(i), split, msb);
            // raw chunks, least significant first: the last one the decoder reads (nr - 16 (k - 1) bits, 0 bits without raw bits,
            // which leaves x as it is), then 16 bits each
            int c = sp.num_raw - kRawChunk * ((sp.num_raw - 1) / kRawChunk);
            renorm((kStateLow >> c) << 32);
            x = (x << c) | (uint64_t)(sp.raw & ((int64_t(1) << c) - 1));
            for (int at = c; at < sp.num_raw; at += kRawChunk) {
                renorm((kStateLow >> kRawChunk) << 32);
                x = (x << kRawChunk) | (uint64_t)((sp.raw >> at) & ((int64_t(1) << kRawChunk) - 1));
            }
            const EncToken &e = tok[sp.token];
            renorm(e.x_max);
            const uint64_t q = (uint64_t)(((unsigned __int128)(x << 1) * e.rcp) >> 64) >> e.shift;
            x += e.start + q * e.cmpl;
        }
    }
    if (pos < 2) return -1;
    words[--pos] = (uint32_t)x;
    words[--pos] = (uint32_t)(x >> 32);
    return pos;
}

// ---- device: histograms of fine tokens for estimate_stream_bits --------------------------------------------------------------------

constexpr int kEstThreads = 256;
constexpr int kEstBins = (1 << kMaxSplitExp) + (kMaxExponent - kMaxSplitExp + 1);  // msb_bits 0

// per stream: the minimum, and the largest of the shifted values and of the zigzagged differences
__global__ void __launch_bounds__(kEstThreads) estimate_range_kernel(const int count, const int64_t *__restrict__ streams,
                                                                     long long *__restrict__ ranges /* [S][3]: min, max, max zz(diff) */) {
    const int s = blockIdx.y;
    const int64_t *v = streams + (size_t)s * count;
    long long lo = LLONG_MAX, hi = LLONG_MIN, dz = 0;
    for (int i = blockIdx.x * kEstThreads + threadIdx.x; i < count; i += gridDim.x * kEstThreads) {
        const int64_t x = v[i];
        lo = min(lo, (long long)x), hi = max(hi, (long long)x);
        dz = max(dz, (long long)zigzag(x - (i > 0 ? v[i - 1] : 0)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        dz = max(dz, __shfl_xor_sync(0xffffffffu, dz, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&ranges[3 * s], lo);
        atomicMax(&ranges[3 * s + 1], hi);
        atomicMax(&ranges[3 * s + 2], dz);
    }
}

// per stream and mapping (0: shifted to the minimum, 1: zigzagged differences): the histogram of tokens with split_exp the bit length of
// the largest mapped value (at most kMaxSplitExp) and no leading bits
__global__ void __launch_bounds__(kEstThreads) estimate_hist_kernel(const int count, const int64_t *__restrict__ streams,
                                                                    const long long *__restrict__ ranges, unsigned *__restrict__ hist) {
    __shared__ unsigned local[kEstBins];
    const int s = blockIdx.y >> 1, mapping = blockIdx.y & 1;
    for (int b = threadIdx.x; b < kEstBins; b += kEstThreads) local[b] = 0u;
    __syncthreads();
    const int64_t *v = streams + (size_t)s * count;
    const long long lo = ranges[3 * s];
    const int64_t vmax = mapping ? ranges[3 * s + 2] : (int64_t)(ranges[3 * s + 1] - lo);
    const int split = min(bits_of(vmax), kMaxSplitExp);
    for (int i = blockIdx.x * kEstThreads + threadIdx.x; i < count; i += gridDim.x * kEstThreads) {
        const int64_t m = mapping ? zigzag(v[i] - (i > 0 ? v[i - 1] : 0)) : v[i] - lo;
        atomicAdd(&local[split_value(m, split, 0).token], 1u);
    }
    __syncthreads();
    unsigned *out = hist + (size_t)blockIdx.y * kEstBins;
    for (int b = threadIdx.x; b < kEstBins; b += kEstThreads)
        if (local[b]) atomicAdd(&out[b], local[b]);
}

}  // namespace

extern "C" {

size_t igs_rans_payload_bound(int num_streams, int64_t count) {
    // a token symbol and at most four raw chunks per value, each at most one 32-bit word, and the final state
    return 4 * (size_t)(num_streams > 0 ? num_streams : 0) * (size_t)(count > 0 ? count : 0) * 5 + 8;
}

int igs_rans_encode(int num_streams, int64_t count, const int64_t *streams, int num_threads, uint8_t *payload, size_t payload_capacity,
                    size_t *payload_bytes, int64_t *models, int64_t *codes, double *payload_bits) {
    const char *who = "igs_rans_encode";
    IGS_REQUIRE(num_streams >= 1 && count >= 1, "%s: streams must be non-empty", who);
    IGS_REQUIRE(streams && payload && payload_bytes && models && codes && payload_bits, "%s: null pointer", who);
    const size_t n = (size_t)count;
    // the four mappings of every stream (raw values or differences, shift or zigzag), fitted on host threads
    std::vector<Fit> fits(4 * (size_t)num_streams);
    parallel_for(fits.size(), [&](size_t t) { fits[t] = fit_one(streams + (t / 4) * n, n, (t >> 1) & 1, t & 1); }, num_threads);
    auto pick = [&](size_t a, size_t b) -> const Fit & { return fits[b].bits < fits[a].bits ? fits[b] : fits[a]; };

    std::vector<Mapping> mapped(num_streams);
    std::vector<std::vector<EncToken>> tokens(num_streams);
    std::vector<int> split(num_streams), msb(num_streams);
    for (int s = 0; s < num_streams; ++s) {
        const Fit &raw = pick(4 * s, 4 * s + 1), &diff = pick(4 * s + 2, 4 * s + 3);
        const bool delta = diff.bits < raw.bits;
        const Fit &f = delta ? diff : raw;
        const TokenModel &m = f.model;
        if ((int)m.codes.size() > kMaxTokens) return igs::set_error(IGS_ERR_INVALID, "%s: more than %d tokens", who, kMaxTokens);
        mapped[s] = Mapping{streams + (size_t)s * n, delta, f.zigzag_mapped, f.param}, tokens[s] = encoder_tokens(m.freqs), split[s] = m.split_exp, msb[s] = m.msb_bits;
        int64_t *row = models + (size_t)s * IGS_RANS_MODEL_FIELDS;
        row[0] = delta, row[1] = f.zigzag_mapped, row[2] = f.param, row[3] = m.split_exp, row[4] = m.msb_bits, row[5] = m.mantissa_bits;
        row[6] = (int64_t)m.codes.size();
        std::copy(m.codes.begin(), m.codes.end(), codes + (size_t)s * kMaxTokens);
        payload_bits[s] = m.payload_bits;
    }
    // the words go backward into the caller's buffer, then to its start (little-endian words, the byte order of the format)
    static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "the payload is written as host words");
    const int64_t capacity = (int64_t)(payload_capacity / 4);
    std::unique_ptr<uint32_t[]> words(new uint32_t[capacity > 0 ? capacity : 1]);
    const int64_t first = rans_pack(mapped, n, tokens, split.data(), msb.data(), words.get(), capacity);
    IGS_REQUIRE(first >= 0, "%s: the payload exceeds the capacity of %zu bytes", who, payload_capacity);
    *payload_bytes = 4 * (size_t)(capacity - first);
    memcpy(payload, words.get() + first, *payload_bytes);
    return IGS_OK;
}

int igs_rans_decode(int num_streams, int64_t count, const int64_t *models, const int64_t *codes, const uint8_t *payload,
                    size_t payload_size, int64_t *values) {
    const char *who = "igs_rans_decode";
    IGS_REQUIRE(num_streams >= 0 && count >= 0, "%s: negative size", who);
    IGS_REQUIRE(payload && (num_streams == 0 || (models && codes && values)), "%s: null pointer", who);
    IGS_REQUIRE(payload_size % 4 == 0 && payload_size >= 8, "%s: invalid rANS payload", who);
    const size_t num_words = payload_size / 4;
    auto word = [payload](size_t k) {  // little-endian words (the static_assert of the encoder)
        uint32_t w;
        memcpy(&w, payload + 4 * k, 4);
        return w;
    };
    // per stream: the token of each slot of the state's low kPrec bits (16-bit entries: the table stays in the core's cache) and each
    // token's frequency, first slot, smallest value and raw-bit count
    struct Tok {
        uint32_t freq, start;
        int64_t base;
        int num_raw;
    };
    struct Table {
        std::vector<uint16_t> slot;
        std::vector<Tok> tok;
    };
    std::vector<Table> tables(num_streams);
    for (int s = 0; s < num_streams; ++s) {
        const int64_t *row = models + (size_t)s * IGS_RANS_MODEL_FIELDS;
        const int split = (int)row[3], msb = (int)row[4], mb = (int)row[5];
        const int64_t num_codes = row[6];
        IGS_REQUIRE(split >= 0 && split <= 62 && msb >= 0 && msb <= split && mb >= 0 && mb <= 3 && num_codes >= 1 && num_codes <= kMaxTokens,
                    "%s: invalid token model of stream %d", who, s);
        const int64_t last = num_codes - 1;
        IGS_REQUIRE(!(last >= (int64_t(1) << split) && split + ((last - (int64_t(1) << split)) >> msb) > kMaxExponent),
                    "%s: invalid token model of stream %d", who, s);
        I64 weights(num_codes), freqs;
        for (int64_t k = 0; k < num_codes; ++k)
            IGS_REQUIRE(code_to_weight(codes[(size_t)s * kMaxTokens + k], mb, weights[k]), "%s: invalid token count code", who);
        IGS_REQUIRE(frequencies(weights, freqs), "%s: cannot normalize the token histogram of stream %d", who, s);
        Table &t = tables[s];
        t.slot.resize(size_t(1) << kPrec);
        t.tok.resize(num_codes);
        uint32_t start = 0;
        for (int64_t k = 0; k < num_codes; ++k) {
            Tok &o = t.tok[k];
            token_base(k, split, msb, o.base, o.num_raw);
            o.freq = (uint32_t)freqs[k], o.start = start;
            std::fill(t.slot.begin() + start, t.slot.begin() + start + o.freq, (uint16_t)k);
            start += o.freq;
        }
    }
    uint64_t x = ((uint64_t)word(0) << 32) | word(1);
    size_t pos = 2;
    for (int s = 0; s < num_streams; ++s) {
        const uint16_t *slot = tables[s].slot.data();
        const Tok *tok = tables[s].tok.data();
        int64_t *out = values + (size_t)s * (size_t)count;
        for (int64_t i = 0; i < count; ++i) {
            const uint32_t sl = (uint32_t)(x & ((uint64_t(1) << kPrec) - 1));
            const Tok &o = tok[slot[sl]];
            x = (uint64_t)o.freq * (x >> kPrec) + sl - o.start;
            if (x < kStateLow) {
                IGS_REQUIRE(pos < num_words, "%s: truncated rANS payload", who);
                x = (x << 32) | word(pos++);
            }
            int64_t raw = 0;
            for (int left = o.num_raw; left > 0;) {
                const int chunk = std::min(left, kRawChunk);
                left -= chunk;
                raw = (raw << chunk) | (int64_t)(x & ((uint64_t(1) << chunk) - 1));
                x >>= chunk;
                if (x < kStateLow) {
                    IGS_REQUIRE(pos < num_words, "%s: truncated rANS payload", who);
                    x = (x << 32) | word(pos++);
                }
            }
            out[i] = o.base | raw;
        }
    }
    return IGS_OK;
}

size_t igs_estimate_bits_workspace(int num_streams) {
    return 256 + sizeof(unsigned) * (size_t)kEstBins * 2 * (size_t)(num_streams > 0 ? num_streams : 0) +
           sizeof(long long) * 3 * (size_t)(num_streams > 0 ? num_streams : 0);
}

int igs_estimate_stream_bits(int num_streams, int64_t count, const int64_t *streams, double *bits, void *workspace, size_t workspace_bytes,
                             void *stream) {
    const char *who = "igs_estimate_stream_bits";
    IGS_REQUIRE(num_streams >= 1 && count >= 1 && count <= INT32_MAX, "%s: streams must be non-empty (and below 2^31 values)", who);
    IGS_REQUIRE(streams && bits && workspace, "%s: null pointer", who);
    IGS_REQUIRE(workspace_bytes >= igs_estimate_bits_workspace(num_streams), "%s: workspace too small", who);
    IGS_REQUIRE(igs::aligned(workspace, 16) && igs::aligned(streams, 8), "%s: misaligned pointer", who);
    cudaStream_t s = igs::as_stream(stream);
    long long *ranges = static_cast<long long *>(workspace);
    unsigned *hist = reinterpret_cast<unsigned *>(static_cast<char *>(workspace) + 256 + sizeof(long long) * 3 * (size_t)num_streams);
    std::vector<long long> init(3 * (size_t)num_streams);
    for (int k = 0; k < num_streams; ++k) init[3 * k] = LLONG_MAX, init[3 * k + 1] = LLONG_MIN, init[3 * k + 2] = 0;
    const size_t hist_bytes = sizeof(unsigned) * (size_t)kEstBins * 2 * num_streams;
    if (cudaMemcpyAsync(ranges, init.data(), sizeof(long long) * init.size(), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemsetAsync(hist, 0, hist_bytes, s) != cudaSuccess)
        return igs::check_launch(who);
    const int blocks = std::min(igs::ceil_div((int)count, kEstThreads), 64);
    estimate_range_kernel<<<dim3(blocks, num_streams), kEstThreads, 0, s>>>((int)count, streams, ranges);
    estimate_hist_kernel<<<dim3(blocks, 2 * num_streams), kEstThreads, 0, s>>>((int)count, streams, ranges, hist);
    std::vector<unsigned> h((size_t)kEstBins * 2 * num_streams);
    std::vector<long long> r(3 * (size_t)num_streams);
    if (cudaMemcpyAsync(h.data(), hist, hist_bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(r.data(), ranges, sizeof(long long) * r.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return igs::check_launch(who);
    // the reference's formula: per mapping and split_exp, the entropy of the token counts, the raw bits and kEstimateTableBits per
    // used token; the smallest over both mappings and every split_exp
    I64 fine, counts;
    std::vector<double> terms;
    for (int k = 0; k < num_streams; ++k) {
        double best = INFINITY;
        for (int mapping = 0; mapping < 2; ++mapping) {
            const int64_t vmax = mapping ? r[3 * k + 2] : (int64_t)(r[3 * k + 1] - r[3 * k]);
            const int split = std::min(bits_of(vmax), kMaxSplitExp);
            const unsigned *src = h.data() + (size_t)(2 * k + mapping) * kEstBins;
            size_t used = 0;
            for (size_t b = 0; b < (size_t)kEstBins; ++b)
                if (src[b]) used = b + 1;
            fine.assign(src, src + used);
            const std::vector<FineBin> bins = fine_bins(fine, split, 0);
            for (int sp = 0; sp <= split; ++sp) {
                const int64_t raw_bits = coarsen(bins, sp, 0, counts);
                terms.clear();
                for (int64_t c : counts)
                    if (c > 0) terms.push_back((double)c * std::log2((double)count / (double)c));
                const double est = numpy_sum(terms.data(), terms.size()) + (double)raw_bits + (double)(kEstimateTableBits * (int64_t)terms.size());
                best = std::min(best, est);
            }
        }
        bits[k] = best;
    }
    return IGS_OK;
}

}  // extern "C"
