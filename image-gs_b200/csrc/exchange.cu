// Exchange of the tile-row bands' partial gradients over peer memory (NVLink through NVSwitch), one process per GPU of one machine.
//
// With one image split into tile-row bands, every rank ends its band's raster step holding partial sums of v_xy, v_conic, v_colors and the
// loss over all N Gaussians; the parameter gradients need their sum over the ranks followed by the projection backward. Instead of an
// all-reduce followed by every rank repeating the projection backward on all N Gaussians, each rank takes one share of the Gaussians:
//   band_reduce_kernel: announce "my partials are complete" to every rank, wait for every rank's announcement, then for each Gaussian of
//                       this rank's share read its partials from every rank's memory (plain peer loads), add them in rank order, run the
//                       projection backward and store the results into every rank's results buffer (plain peer stores); the last of
//                       its blocks to finish (a ticket in the rank's own words) announces "my share is written" to every rank and waits
//                       for every rank's announcement: the results buffer is then complete on this rank. One kernel per step; no block
//                       waits for another block of its own launch.
// Per rank and step this moves (world - 1) / world of the partials in and of the results out over NVLink, with two rank-wide waits. The
// sums are formed by one rank each in a fixed order, so every rank holds bit-identical gradients.
//
// Synchronisation words (per rank, in its exchange buffer, written by the peers with relaxed stores at system scope, polled with relaxed
// loads and read once more with acquire loads): ready[q] and done[q] hold the last step for which rank q announced; step counts this
// rank's completed exchanges. Every wait polls with a deadline (%globaltimer) and, past it, records IGS_BAND_TIMEOUT_* in the rank's
// error word and returns without touching peer data, so a missing rank makes the step fail instead of hanging the GPU. The ranks' kernels never wait on one another on one GPU:
// each rank is its own GPU.
//
// The buffers are exported and mapped with CUDA IPC (igs_ipc_export / igs_ipc_open): an allocation is exported whole, so the offset of
// the exchange buffer inside it travels with the handle.
#include <algorithm>
#include <cstddef>
#include <cstring>

#include "igs_common.cuh"
#include "project_math.cuh"

namespace {

constexpr int kMaxRanks = IGS_MAX_BAND_RANKS;
constexpr int kThreads = 256;

struct SyncWords {
    unsigned ready[kMaxRanks];
    unsigned done[kMaxRanks];
    unsigned step;
    unsigned error;
    unsigned ticket;  // blocks of this rank's band_reduce_kernel that have finished this step (this rank's own; zero between steps)
    unsigned pad[IGS_BAND_SYNC_WORDS - 2 * kMaxRanks - 3];
};
static_assert(sizeof(SyncWords) == IGS_BAND_SYNC_WORDS * sizeof(unsigned), "sync word layout");
static_assert(offsetof(SyncWords, step) == IGS_BAND_SYNC_STEP * sizeof(unsigned), "sync word layout");
static_assert(offsetof(SyncWords, error) == IGS_BAND_SYNC_ERROR * sizeof(unsigned), "sync word layout");

struct Peers {
    const float *partials[kMaxRanks];
    float *results[kMaxRanks];
    SyncWords *sync[kMaxRanks];
};

// Synchronisation with the other ranks: relaxed stores of the flags, relaxed polling, then one acquire load per flag; the stores a flag
// announces are fenced (release, system scope) by the blocks that made them. System-scope fences cost microseconds each, so the protocol
// has one per block of band_reduce_kernel and none in the waits.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ unsigned load_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_relaxed_sys(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned load_relaxed_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// a peer's values, fetched from its memory (no stale line from an earlier step in this SM's L1)
__device__ __forceinline__ float load_peer(const float *p) {
    float v;
    asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float2 load_peer2(const float *p) {
    float2 v;
    asm volatile("ld.volatile.global.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Announce `value` in slot `rank` of every rank's words (ready or done), then wait until every rank's announcement in this rank's own
// words reaches `value`. One thread. Returns false (and records `code` in the error word) past the deadline.
__device__ bool announce_and_wait(const Peers &peers, const int world, const int rank, const bool done_words, const unsigned value,
                                  const unsigned long long timeout_ns, const unsigned code) {
    // No fence here: what the ready flags announce was written by kernels that have completed (the band's raster step), and the
    // done flags are announced by band_reduce_kernel's last block after the fences that order every block's stores before them
    for (int q = 0; q < world; ++q) {
        SyncWords *w = peers.sync[q];
        store_relaxed_sys(done_words ? &w->done[rank] : &w->ready[rank], value);
    }
    SyncWords *me = peers.sync[rank];
    const unsigned *words = done_words ? me->done : me->ready;
    const unsigned long long deadline = global_ns() + timeout_ns;
    for (int q = 0; q < world; ++q) {
        // the counters only grow; a difference of at most 2^31 compares steps across a wrap of the 32-bit count
        while ((int)(load_relaxed_sys(&words[q]) - value) < 0) {
            if (global_ns() > deadline) {
                atomicOr(&me->error, code);
                return false;
            }
            __nanosleep(64);
        }
    }
    // acquire: the data each rank wrote before its flag is read after it
    for (int q = 0; q < world; ++q) (void)load_acquire_sys(&words[q]);
    return true;
}

// Results layout of a rank: v_cov2d [N,3], v_mean2d [N,2], v_scale [N,2], v_rot [N], v_colors [N,C], loss
struct ResultsLayout {
    size_t cov, mean, scale, rot, colors, loss;
    __host__ __device__ ResultsLayout(size_t n, int c)
        : cov(0), mean(3 * n), scale(5 * n), rot(7 * n), colors(8 * n), loss((8 + (size_t)c) * n) {}
};

// One Gaussian's partials from kGroup ranks, every load issued before the first addition (peer loads take an NVLink round trip each)
template <int kMaxC, int kGroup>
__device__ __forceinline__ void add_partials(const Peers &peers, const int q0, const int world, const size_t nn, const int g,
                                             const int channels, float (&vxy)[2], float (&vcon)[3], float (&vcol)[kMaxC]) {
    float t[kGroup][5 + kMaxC];
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
        if (q0 + j >= world) continue;
        const float *p = peers.partials[q0 + j];
        const float2 xy = load_peer2(p + 2 * (size_t)g);
        t[j][0] = xy.x;
        t[j][1] = xy.y;
#pragma unroll
        for (int k = 0; k < 3; ++k) t[j][2 + k] = load_peer(p + 2 * nn + 3 * (size_t)g + k);
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) t[j][5 + c] = c < channels ? load_peer(p + 5 * nn + (size_t)g * channels + c) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
        if (q0 + j >= world) continue;
        vxy[0] += t[j][0];
        vxy[1] += t[j][1];
#pragma unroll
        for (int k = 0; k < 3; ++k) vcon[k] += t[j][2 + k];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) vcol[c] += t[j][5 + c];
    }
}

template <int kMaxC>
__global__ void __launch_bounds__(kThreads) band_reduce_kernel(const Peers peers, const int world, const int rank, const int n,
                                                               const int channels, const int share_begin, const int share_end,
                                                               const float2 *__restrict__ scales, const float *__restrict__ rotations,
                                                               const float img_w, const float img_h, const int *__restrict__ radii,
                                                               const float *__restrict__ conics, const unsigned long long timeout_ns) {
    constexpr int kGroup = kMaxC <= 4 ? kMaxRanks : 2;  // ranks whose loads are in flight together (registers: kGroup (5 + kMaxC))
    igs::wait_for_predecessor_only();  // this rank's partials are complete (the band's raster step ran before this kernel)
    __shared__ int s_go;
    SyncWords *me = peers.sync[rank];
    if (threadIdx.x == 0) {
        bool go = atomicOr(&me->error, 0u) == 0u;  // a rank that failed an earlier wait stays stopped
        if (go) go = announce_and_wait(peers, world, rank, false, *(volatile unsigned *)&me->step + 1u, timeout_ns, IGS_BAND_TIMEOUT_READY);
        s_go = go ? 1 : 0;
    }
    __syncthreads();

    const size_t nn = (size_t)n;
    const ResultsLayout out(nn, channels);
    const int g = share_begin + blockIdx.x * kThreads + threadIdx.x;
    if (s_go && g < share_end) {
        // the sums in rank order (the same on every rank: each Gaussian is summed by one rank only)
        float vxy[2] = {0.f, 0.f}, vcon[3] = {0.f, 0.f, 0.f}, vcol[kMaxC];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) vcol[c] = 0.f;
        for (int q0 = 0; q0 < world; q0 += kGroup) add_partials<kMaxC, kGroup>(peers, q0, world, nn, g, channels, vxy, vcon, vcol);
        igs::ProjectionGrad pg;
        if (__ldg(&radii[g]) > 0) {
            pg = igs::projection_grad(__ldg(&scales[g]), __ldg(&rotations[g]), img_w, img_h, conics + 3 * (size_t)g, vcon,
                                      make_float2(vxy[0], vxy[1]));
        } else {
            pg.cov2d[0] = pg.cov2d[1] = pg.cov2d[2] = 0.f;
            pg.mean2d = pg.scale = make_float2(0.f, 0.f);
            pg.rot = 0.f;
        }
        for (int q = 0; q < world; ++q) {
            float *r = peers.results[q];
#pragma unroll
            for (int k = 0; k < 3; ++k) r[out.cov + 3 * (size_t)g + k] = pg.cov2d[k];
            r[out.mean + 2 * (size_t)g] = pg.mean2d.x;
            r[out.mean + 2 * (size_t)g + 1] = pg.mean2d.y;
            r[out.scale + 2 * (size_t)g] = pg.scale.x;
            r[out.scale + 2 * (size_t)g + 1] = pg.scale.y;
            r[out.rot + g] = pg.rot;
#pragma unroll
            for (int c = 0; c < kMaxC; ++c)
                if (c < channels) r[out.colors + (size_t)g * channels + c] = vcol[c];
        }
    }
    if (s_go && blockIdx.x == 0 && threadIdx.x == 0) {
        // the loss: every rank adds the partial losses in rank order into its own results
        float loss = 0.f;
        for (int q = 0; q < world; ++q) loss += load_peer(peers.partials[q] + (5 + (size_t)channels) * nn);
        peers.results[rank][out.loss] = loss;
    }
    // The block's peer stores are performed at system scope before its ticket: the barrier orders every thread's stores before thread
    // 0's fence, which is cumulative over them. Every block takes a ticket (also one that did nothing after a failed wait), and the
    // last one, after a fence that orders the others' fenced stores before its own operations, announces "share written" to every
    // rank and waits for every rank's announcement, then counts the step.
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        if (atomicAdd(&me->ticket, 1u) == gridDim.x - 1) {
            fence_acq_rel_sys();
            me->ticket = 0u;  // every block of this step has taken its ticket
            if (atomicOr(&me->error, 0u) == 0u) {
                const unsigned value = *(volatile unsigned *)&me->step + 1u;
                if (announce_and_wait(peers, world, rank, true, value, timeout_ns, IGS_BAND_TIMEOUT_DONE))
                    *(volatile unsigned *)&me->step = value;
            }
        }
    }
}

using GetAddressRange = int (*)(unsigned long long *base, size_t *size, unsigned long long dptr);

// cuMemGetAddressRange of the driver API, through the runtime's entry-point query (no link-time dependency on libcuda)
GetAddressRange address_range_fn() {
    static GetAddressRange fn = nullptr;
    if (fn == nullptr) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetAddressRange>(p);
    }
    return fn;
}

}  // namespace

extern "C" {

size_t igs_band_sync_bytes(void) { return sizeof(SyncWords); }

size_t igs_band_results_floats(int num_points, int channels) {
    return (size_t)(num_points > 0 ? num_points : 0) * (8 + (size_t)(channels > 0 ? channels : 0)) + 1;
}

int igs_ipc_export(const void *dev_ptr, void *handle, uint64_t *offset) {
    IGS_REQUIRE(dev_ptr && handle && offset, "igs_ipc_export: null pointer");
    const GetAddressRange range = address_range_fn();
    if (range == nullptr) return igs::set_error(IGS_ERR_CUDA, "igs_ipc_export: cuMemGetAddressRange is unavailable");
    unsigned long long base = 0;
    size_t size = 0;
    if (range(&base, &size, (unsigned long long)(uintptr_t)dev_ptr) != 0)
        return igs::set_error(IGS_ERR_INVALID, "igs_ipc_export: %p is not device memory of the current context", dev_ptr);
    cudaIpcMemHandle_t h;
    const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "igs_ipc_export: %s", cudaGetErrorString(err));
    static_assert(sizeof(h) == IGS_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *offset = (uint64_t)((uintptr_t)dev_ptr - (uintptr_t)base);
    return IGS_OK;
}

int igs_ipc_open(const void *handle, uint64_t offset, void **dev_ptr) {
    IGS_REQUIRE(handle && dev_ptr, "igs_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "igs_ipc_open: %s", cudaGetErrorString(err));
    *dev_ptr = static_cast<char *>(base) + offset;
    return IGS_OK;
}

int igs_ipc_close(void *dev_ptr, uint64_t offset) {
    IGS_REQUIRE(dev_ptr != nullptr, "igs_ipc_close: null pointer");
    const cudaError_t err = cudaIpcCloseMemHandle(static_cast<char *>(dev_ptr) - offset);
    if (err != cudaSuccess) return igs::set_error(IGS_ERR_CUDA, "igs_ipc_close: %s", cudaGetErrorString(err));
    return IGS_OK;
}

int igs_band_reduce(int world, int rank, int num_points, int channels, const float *const *partials, float *const *results,
                    void *const *sync, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                    const float *conics, int timeout_ms, void *stream) {
    const char *who = "igs_band_reduce";
    IGS_REQUIRE(world >= 1 && world <= kMaxRanks, "%s: 1 to %d ranks (got %d)", who, kMaxRanks, world);
    IGS_REQUIRE(rank >= 0 && rank < world, "%s: rank %d of %d", who, rank, world);
    IGS_REQUIRE(num_points >= 0 && channels >= 0 && channels <= igs::kMaxChannels, "%s: bad sizes", who);
    IGS_REQUIRE(timeout_ms > 0, "%s: the timeout must be positive", who);
    IGS_REQUIRE(partials && results && sync, "%s: null pointer arrays", who);
    IGS_REQUIRE(num_points == 0 || (scales2d && rotation && radii && conics), "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || igs::aligned(scales2d, 8), "%s: scales2d must be 8-byte aligned", who);
    Peers peers;
    memset(&peers, 0, sizeof(peers));
    for (int q = 0; q < world; ++q) {
        IGS_REQUIRE(partials[q] && results[q] && sync[q], "%s: null pointer for rank %d", who, q);
        IGS_REQUIRE(igs::aligned(sync[q], 16), "%s: the sync words of rank %d must be 16-byte aligned", who, q);
        peers.partials[q] = partials[q];
        peers.results[q] = results[q];
        peers.sync[q] = static_cast<SyncWords *>(sync[q]);
    }
    const int share_begin = (int)((int64_t)num_points * rank / world), share_end = (int)((int64_t)num_points * (rank + 1) / world);
    const int blocks = std::max(1, igs::ceil_div(share_end - share_begin, kThreads));
    const unsigned long long timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
    cudaStream_t s = igs::as_stream(stream);
    const auto kernel = channels <= 4 ? band_reduce_kernel<4> : band_reduce_kernel<igs::kMaxChannels>;
    igs::launch(kernel, blocks, kThreads, 0, s, peers, world, rank, num_points, channels, share_begin, share_end,
                reinterpret_cast<const float2 *>(scales2d), rotation, (float)img_width, (float)img_height, radii, conics, timeout_ns);
    return igs::check_launch(who);
}

}  // extern "C"
