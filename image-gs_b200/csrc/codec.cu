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

// the histogram of a coarser tokenizer (split_exp <= fine_split, msb_bits <= fine_msb) from a fine one: every value of a fine token has
// the same coarse token and raw-bit count, those of the fine token's smallest value. Returns the raw bits.
int64_t coarsen(const I64 &fine, int fine_split, int fine_msb, int split_exp, int msb_bits, I64 &counts) {
    counts.clear();
    int64_t raw_bits = 0;
    for (size_t t = 0; t < fine.size(); ++t) {
        if (fine[t] == 0) continue;
        int64_t base;
        int nr;
        token_base((int64_t)t, fine_split, fine_msb, base, nr);
        const Split sp = split_value(base, split_exp, msb_bits);
        if (sp.token >= (int64_t)counts.size()) counts.resize(sp.token + 1, 0);
        counts[sp.token] += fine[t];
        raw_bits += fine[t] * sp.num_raw;
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
    TokenModel best;
    bool have = false;
    I64 counts, codes, weights, freqs;
    std::vector<double> terms;
    for (int split = 0; split <= fine_split; ++split) {
        for (int msb = 0; msb <= std::min(split, kMaxMsbBits); ++msb) {
            const int64_t raw_bits = coarsen(fine, fine_split, fine_msb, split, msb, counts);
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

// int(np.round(np.median(values))): the middle value, or the mean of the two middle ones, rounded half to even
int64_t median_rounded(I64 v) {
    const size_t half = v.size() / 2;
    std::nth_element(v.begin(), v.begin() + half, v.end());
    double m = (double)v[half];
    if (v.size() % 2 == 0) m = ((double)*std::max_element(v.begin(), v.begin() + half) + m) / 2.0;
    return (int64_t)std::nearbyint(m);
}

struct Fit {
    double bits = 0.0;
    bool zigzag_mapped = false;
    int64_t param = 0;
    I64 mapped;
    TokenModel model;
};

// The cheaper mapping of a stream to non-negative integers (shift to the minimum first, then zigzag around the median) with its model
Fit fit_mapping(const I64 &values) {
    Fit best;
    for (int zz = 0; zz < 2; ++zz) {
        const int64_t param = zz ? median_rounded(values) : *std::min_element(values.begin(), values.end());
        I64 mapped(values.size());
        int64_t vmax = 0;
        for (size_t i = 0; i < values.size(); ++i) {
            mapped[i] = zz ? zigzag(values[i] - param) : values[i] - param;
            vmax = std::max(vmax, mapped[i]);
        }
        int split, msb;
        fine_tokenizer(vmax, split, msb);
        I64 fine;
        for (int64_t m : mapped) {
            const int64_t t = split_value(m, split, msb).token;
            if (t >= (int64_t)fine.size()) fine.resize(t + 1, 0);
            ++fine[t];
        }
        TokenModel model = best_model(fine, split, msb, (int64_t)values.size());
        const double bits = (double)(1 + exp_golomb_bits(zigzag(param))) + model.bits;
        if (!zz || bits < best.bits) {
            best.bits = bits, best.zigzag_mapped = zz == 1, best.param = param;
            best.mapped = std::move(mapped);
            best.model = std::move(model);
        }
    }
    return best;
}

struct Symbol {
    uint32_t start, freq;
    int prec;
};

// rANS over symbols given in decoding order (encoded last to first); 32-bit words, the last emitted first, little-endian
std::vector<uint8_t> rans_pack(const std::vector<Symbol> &symbols) {
    uint64_t x = kStateLow;
    std::vector<uint32_t> out;
    for (size_t k = symbols.size(); k-- > 0;) {
        const Symbol &s = symbols[k];
        if (x >= ((kStateLow >> s.prec) << 32) * (uint64_t)s.freq) {
            out.push_back((uint32_t)x);
            x >>= 32;
        }
        x = ((x / s.freq) << s.prec) + x % s.freq + s.start;
    }
    out.push_back((uint32_t)x);
    out.push_back((uint32_t)(x >> 32));
    std::vector<uint8_t> bytes(4 * out.size());
    for (size_t i = 0; i < out.size(); ++i) {
        const uint32_t w = out[out.size() - 1 - i];
        for (int b = 0; b < 4; ++b) bytes[4 * i + b] = (uint8_t)(w >> (8 * b));
    }
    return bytes;
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
    // candidates: raw values and differences of every stream, fitted on host threads
    std::vector<I64> cand(2 * (size_t)num_streams);
    for (int s = 0; s < num_streams; ++s) {
        const int64_t *v = streams + (size_t)s * n;
        cand[2 * s].assign(v, v + n);
        I64 &d = cand[2 * s + 1];
        d.resize(n);
        for (size_t i = 0; i < n; ++i) d[i] = v[i] - (i > 0 ? v[i - 1] : 0);
    }
    std::vector<Fit> fits(cand.size());
    std::atomic<size_t> next{0};
    auto work = [&]() {
        for (size_t t = next++; t < cand.size(); t = next++) fits[t] = fit_mapping(cand[t]);
    };
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>(cand.size(), num_threads > 0 ? (size_t)num_threads : hw);
    std::vector<std::thread> pool;
    for (size_t t = 1; t < threads; ++t) pool.emplace_back(work);
    work();
    for (std::thread &t : pool) t.join();

    std::vector<Symbol> symbols;
    symbols.reserve(n * num_streams * 2);
    for (int s = 0; s < num_streams; ++s) {
        const bool delta = fits[2 * s + 1].bits < fits[2 * s].bits;
        const Fit &f = fits[2 * s + (delta ? 1 : 0)];
        const TokenModel &m = f.model;
        if ((int)m.codes.size() > kMaxTokens) return igs::set_error(IGS_ERR_INVALID, "%s: more than %d tokens", who, kMaxTokens);
        I64 starts(m.freqs.size(), 0);
        for (size_t t = 1; t < starts.size(); ++t) starts[t] = starts[t - 1] + m.freqs[t - 1];
        for (int64_t v : f.mapped) {
            const Split sp = split_value(v, m.split_exp, m.msb_bits);
            symbols.push_back({(uint32_t)starts[sp.token], (uint32_t)m.freqs[sp.token], kPrec});
            for (int left = sp.num_raw; left > 0;) {  // raw bits as uniform symbols, most significant first
                const int chunk = std::min(left, kRawChunk);
                left -= chunk;
                symbols.push_back({(uint32_t)((sp.raw >> left) & ((int64_t(1) << chunk) - 1)), 1u, chunk});
            }
        }
        int64_t *row = models + (size_t)s * IGS_RANS_MODEL_FIELDS;
        row[0] = delta, row[1] = f.zigzag_mapped, row[2] = f.param, row[3] = m.split_exp, row[4] = m.msb_bits, row[5] = m.mantissa_bits;
        row[6] = (int64_t)m.codes.size();
        std::copy(m.codes.begin(), m.codes.end(), codes + (size_t)s * kMaxTokens);
        payload_bits[s] = m.payload_bits;
    }
    const std::vector<uint8_t> bytes = rans_pack(symbols);
    IGS_REQUIRE(bytes.size() <= payload_capacity, "%s: payload of %zu bytes exceeds the capacity %zu", who, bytes.size(), payload_capacity);
    memcpy(payload, bytes.data(), bytes.size());
    *payload_bytes = bytes.size();
    return IGS_OK;
}

int igs_rans_decode(int num_streams, int64_t count, const int64_t *models, const int64_t *codes, const uint8_t *payload,
                    size_t payload_size, int64_t *values) {
    const char *who = "igs_rans_decode";
    IGS_REQUIRE(num_streams >= 0 && count >= 0, "%s: negative size", who);
    IGS_REQUIRE(payload && (num_streams == 0 || (models && codes && values)), "%s: null pointer", who);
    IGS_REQUIRE(payload_size % 4 == 0 && payload_size >= 8, "%s: invalid rANS payload", who);
    const size_t num_words = payload_size / 4;
    std::vector<uint32_t> words(num_words, 0u);
    for (size_t i = 0; i < num_words; ++i)
        for (int b = 0; b < 4; ++b) words[i] |= (uint32_t)payload[4 * i + b] << (8 * b);
    struct Table {
        int split_exp, msb_bits;
        I64 freqs, starts;
        std::vector<uint32_t> token_of_slot;
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
        Table &t = tables[s];
        t.split_exp = split, t.msb_bits = msb;
        I64 weights(num_codes);
        for (int64_t k = 0; k < num_codes; ++k)
            IGS_REQUIRE(code_to_weight(codes[(size_t)s * kMaxTokens + k], mb, weights[k]), "%s: invalid token count code", who);
        IGS_REQUIRE(frequencies(weights, t.freqs), "%s: cannot normalize the token histogram of stream %d", who, s);
        t.starts.assign(num_codes, 0);
        for (int64_t k = 0; k < num_codes; ++k) {
            if (k > 0) t.starts[k] = t.starts[k - 1] + t.freqs[k - 1];
            t.token_of_slot.insert(t.token_of_slot.end(), (size_t)t.freqs[k], (uint32_t)k);
        }
    }
    uint64_t x = ((uint64_t)words[0] << 32) | words[1];
    size_t pos = 2;
    for (int s = 0; s < num_streams; ++s) {
        const Table &t = tables[s];
        int64_t *out = values + (size_t)s * (size_t)count;
        for (int64_t i = 0; i < count; ++i) {
            const uint64_t slot = x & ((uint64_t(1) << kPrec) - 1);
            const uint32_t token = t.token_of_slot[slot];
            x = (uint64_t)t.freqs[token] * (x >> kPrec) + slot - (uint64_t)t.starts[token];
            if (x < kStateLow) {
                IGS_REQUIRE(pos < num_words, "%s: truncated rANS payload", who);
                x = (x << 32) | words[pos++];
            }
            int64_t base;
            int num_raw;
            token_base(token, t.split_exp, t.msb_bits, base, num_raw);
            int64_t raw = 0;
            for (int left = num_raw; left > 0;) {
                const int chunk = std::min(left, kRawChunk);
                left -= chunk;
                raw = (raw << chunk) | (int64_t)(x & ((uint64_t(1) << chunk) - 1));
                x >>= chunk;
                if (x < kStateLow) {
                    IGS_REQUIRE(pos < num_words, "%s: truncated rANS payload", who);
                    x = (x << 32) | words[pos++];
                }
            }
            out[i] = base | raw;
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
            for (int sp = 0; sp <= split; ++sp) {
                const int64_t raw_bits = coarsen(fine, split, 0, sp, 0, counts);
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
