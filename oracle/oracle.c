/*
 * CPU ORACLE — test infrastructure, not product code.
 *
 * A literal scalar C restatement of the reference's 2D Gaussian rasterization hot path (the gsplat fork under gsplat/gsplat/cuda/csrc/ of
 * BaylorMultimediaLab/image-gs). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may call it, as the checker; the product
 * never links or calls it.
 *
 * Numerics: IEEE single precision without contraction (compile with -ffp-contract=off) and libm's expf/sqrtf/cosf/sinf, where the reference
 * is built with --use_fast_math (approximate sqrt, reciprocal, sin/cos and __expf, FMA contraction). Integer outputs (radii, tile counts,
 * binning, top-K slots) therefore agree with the reference bit for bit except where a float lands within a few ulp of a decision boundary;
 * tests feed each stage the GPU's own previous-stage outputs and report such cases. Two fast-math effects that change integer outcomes far
 * from boundaries are emulated: alpha values below FLT_MIN are flushed to zero (the .ftz of __expf, which makes distant Gaussians tie at
 * exactly 0), and float->int conversions saturate like the GPU's cvt.rzi.
 */
#include <float.h>
#include <limits.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_TILE 16
#define ORC_TOPK 10
#define ORC_EPS 1e-4 /* a double literal in the reference (config.h:9): the forward normalizes in double */
#define ORC_MAX_CHANNELS 12

/* glm-style 2x2 matrix, m[column][row] (helpers.cuh uses glm::mat2, column-major) */
typedef struct {
    float m[2][2];
} mat2;

static mat2 mat2_mul(mat2 a, mat2 b) {
    /* (a*b)[c][r] = a[0][r]*b[c][0] + a[1][r]*b[c][1], the term order of glm's mat2 product */
    mat2 o;
    for (int c = 0; c < 2; ++c)
        for (int r = 0; r < 2; ++r) o.m[c][r] = a.m[0][r] * b.m[c][0] + a.m[1][r] * b.m[c][1];
    return o;
}

static mat2 mat2_transpose(mat2 a) {
    mat2 o;
    o.m[0][0] = a.m[0][0];
    o.m[0][1] = a.m[1][0];
    o.m[1][0] = a.m[0][1];
    o.m[1][1] = a.m[1][1];
    return o;
}

/* rotmat2d (helpers.cuh:265-276): diagonal cos, [0][1] = -sin, [1][0] = sin */
static mat2 rot_matrix(float theta) {
    float c = cosf(theta), s = sinf(theta);
    mat2 r = {{{c, -s}, {s, c}}};
    return r;
}

/* rotmat2d_gradient (helpers.cuh:278-289): diagonal -sin, [0][1] = -cos, [1][0] = cos */
static mat2 rot_matrix_grad(float theta) {
    float c = cosf(theta), s = sinf(theta);
    mat2 r = {{{-s, -c}, {c, -s}}};
    return r;
}

static mat2 diag2(float a, float b) {
    mat2 r = {{{a, 0.f}, {0.f, b}}};
    return r;
}

/* float -> int32 truncation that saturates and maps NaN to 0, as the GPU's cvt.rzi.s32.f32 */
static int cvt_rzi(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT_MAX;
    if (x <= -2147483648.0f) return INT_MIN;
    return (int)x;
}

static int imin_u(int a, int b) { return a < b ? a : b; }

/* Host threads for the parallel loops (orc_set_threads; 1 = scalar) */
static int g_threads = 1;

void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }

int orc_get_threads(void) { return g_threads; }

typedef struct {
    void (*body)(void *ctx, int begin, int end);
    void *ctx;
    int count, chunk;
    int next; /* shared work counter, taken under the mutex */
    pthread_mutex_t lock;
} par_job;

static void *par_worker(void *arg) {
    par_job *job = (par_job *)arg;
    for (;;) {
        pthread_mutex_lock(&job->lock);
        int begin = job->next;
        job->next += job->chunk;
        pthread_mutex_unlock(&job->lock);
        if (begin >= job->count) break;
        int end = begin + job->chunk < job->count ? begin + job->chunk : job->count;
        job->body(job->ctx, begin, end);
    }
    return NULL;
}

/* body(ctx, begin, end) over [0, count) in chunks, on g_threads threads (the calling thread included) */
static void parallel_for(int count, int chunk, void (*body)(void *, int, int), void *ctx) {
    if (g_threads <= 1 || count <= chunk) {
        body(ctx, 0, count);
        return;
    }
    par_job job = {body, ctx, count, chunk, 0, PTHREAD_MUTEX_INITIALIZER};
    int extra = g_threads - 1;
    pthread_t *tids = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)extra);
    int started = 0;
    for (int t = 0; t < extra; ++t)
        if (pthread_create(&tids[t], NULL, par_worker, &job) == 0) ++started;
    par_worker(&job);
    for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
    free(tids);
}

/* get_bbox + get_tile_bbox (helpers.cuh:11-43): tile rectangle [min, max) of a pixel center and pixel radius, clamped to the tile grid */
static void tile_bbox(float cx, float cy, float radius, int tiles_x, int tiles_y, int *x0, int *y0, int *x1, int *y1) {
    float tcx = cx / (float)ORC_TILE, tcy = cy / (float)ORC_TILE;
    float trx = radius / (float)ORC_TILE, try_ = radius / (float)ORC_TILE;
    int a = cvt_rzi(tcx - trx), b = cvt_rzi(tcx + trx + 1), c = cvt_rzi(tcy - try_), d = cvt_rzi(tcy + try_ + 1);
    *x0 = imin_u(a > 0 ? a : 0, tiles_x);
    *x1 = imin_u(b > 0 ? b : 0, tiles_x);
    *y0 = imin_u(c > 0 ? c : 0, tiles_y);
    *y1 = imin_u(d > 0 ? d : 0, tiles_y);
}

/*
 * Projection forward: project_gaussians_2d_scale_rot_forward_kernel (foward2d.cu:9-59) with compute_cov2d_bounds (helpers.cuh:45-68).
 * Outputs must be zero-initialized by the caller (bindings.cu:809-816 allocates them with torch::zeros); Gaussians with a zero determinant
 * keep xys/conics at zero and radius/num_tiles_hit at 0.
 */
void orc_project_fwd(int n, const float *means, const float *scales, const float *rot, int img_h, int img_w, int tiles_x, int tiles_y,
                     float *xys, int *radii, float *conics, int *num_tiles_hit) {
    for (int i = 0; i < n; ++i) {
        radii[i] = 0;
        num_tiles_hit[i] = 0;
        float cx = means[2 * i] * (float)img_w, cy = means[2 * i + 1] * (float)img_h;
        mat2 R = rot_matrix(rot[i]);
        mat2 S = diag2(scales[2 * i], scales[2 * i + 1]);
        mat2 M = mat2_mul(R, S);
        mat2 cov = mat2_mul(M, mat2_transpose(M));
        float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[1][1];
        float det = a * c - b * b;
        if (det == 0.f) continue;
        float inv_det = 1.f / det;
        float bm = 0.5f * (a + c);
        float v1 = bm + sqrtf(fmaxf(0.1f, bm * bm - det));
        float v2 = bm - sqrtf(fmaxf(0.1f, bm * bm - det));
        float radius = ceilf(3.f * sqrtf(fmaxf(v1, v2)));
        conics[3 * i] = c * inv_det;
        conics[3 * i + 1] = -b * inv_det;
        conics[3 * i + 2] = a * inv_det;
        xys[2 * i] = cx;
        xys[2 * i + 1] = cy;
        radii[i] = cvt_rzi(radius);
        int x0, y0, x1, y1;
        tile_bbox(cx, cy, radius, tiles_x, tiles_y, &x0, &y0, &x1, &y1);
        int32_t area = (int32_t)((uint32_t)(x1 - x0) * (uint32_t)(y1 - y0));
        if (area > 0) num_tiles_hit[i] = area;
    }
}

/*
 * Projection backward: project_gaussians_2d_scale_rot_backward_kernel (backward2d.cu:53-100) with cov2d_to_conic_vjp (helpers.cuh:71-82),
 * restated literally, including its use of the summed off-diagonal conic gradient and the factor 2 on G_12 (it is not the derivative of
 * the forward with respect to scale and rotation; parity means matching it). Outputs zero-initialized by the caller (bindings.cu:862-869).
 */
void orc_project_bwd(int n, const float *scales, const float *rot, int img_h, int img_w, const int *radii, const float *conics,
                     const float *v_xy, const float *v_conic, float *v_cov2d, float *v_mean2d, float *v_scale, float *v_rot) {
    for (int i = 0; i < n; ++i) {
        if (radii[i] <= 0) continue;
        float x = conics[3 * i], y = conics[3 * i + 1], z = conics[3 * i + 2];
        float gx = v_conic[3 * i], gy = v_conic[3 * i + 1], gz = v_conic[3 * i + 2];
        mat2 X = {{{x, y}, {y, z}}};
        mat2 G = {{{gx, gy}, {gy, gz}}};
        mat2 NX = {{{-x, -y}, {-y, -z}}};
        mat2 V = mat2_mul(mat2_mul(NX, G), X);
        float G11 = V.m[0][0], G12 = V.m[1][0] + V.m[0][1], G22 = V.m[1][1];
        v_cov2d[3 * i] = G11;
        v_cov2d[3 * i + 1] = G12;
        v_cov2d[3 * i + 2] = G22;

        float sx = scales[2 * i], sy = scales[2 * i + 1];
        mat2 R = rot_matrix(rot[i]);
        mat2 Rg = rot_matrix_grad(rot[i]);
        mat2 S = diag2(sx, sy);
        mat2 M = mat2_mul(R, S);
        mat2 t1 = mat2_mul(mat2_mul(Rg, S), mat2_transpose(M));
        mat2 t2 = mat2_mul(mat2_mul(M, mat2_transpose(S)), mat2_transpose(Rg));
        mat2 theta;
        for (int c = 0; c < 2; ++c)
            for (int r = 0; r < 2; ++r) theta.m[c][r] = t1.m[c][r] + t2.m[c][r];
        mat2 sxg = mat2_mul(mat2_mul(R, diag2(2.f * sx, 0.f)), mat2_transpose(R));
        mat2 syg = mat2_mul(mat2_mul(R, diag2(0.f, 2.f * sy)), mat2_transpose(R));
        v_scale[2 * i] = G11 * sxg.m[0][0] + 2.f * G12 * sxg.m[0][1] + G22 * sxg.m[1][1];
        v_scale[2 * i + 1] = G11 * syg.m[0][0] + 2.f * G12 * syg.m[0][1] + G22 * syg.m[1][1];
        v_rot[i] = G11 * theta.m[0][0] + 2.f * G12 * theta.m[0][1] + G22 * theta.m[1][1];
        v_mean2d[2 * i] = v_xy[2 * i] * (float)img_w;
        v_mean2d[2 * i + 1] = v_xy[2 * i + 1] * (float)img_h;
    }
}

/* compute_cumulative_intersects (utils.py:96-115): inclusive int32 prefix sum (wrapping like torch.cumsum in int32) */
void orc_cumsum(int n, const int *in, int *out) {
    uint32_t acc = 0;
    for (int i = 0; i < n; ++i) {
        acc += (uint32_t)in[i];
        out[i] = (int)acc;
    }
}

typedef struct {
    uint32_t key;
    int32_t val;
    int32_t pos;
} keyval;

static int keyval_cmp(const void *pa, const void *pb) {
    const keyval *a = (const keyval *)pa, *b = (const keyval *)pb;
    if (a->key != b->key) return a->key < b->key ? -1 : 1;
    return a->pos < b->pos ? -1 : (a->pos > b->pos); /* stability */
}

/*
 * sort_intersects_by_tile (bindings.cu:106-167): map_intersects_to_tiles (forward.cu:76-105) over capacity slots, a stable sort by tile key
 * (the CUB radix sort of bindings.cu:145-159 is stable; keys of consistent inputs fit its end_bit), and get_tile_bin_edges_from_tiles
 * (forward.cu:109-122). Padding slots carry key num_tiles and value 0. gaussian_ids_sorted has capacity entries; tile_bins [T, 2] zeros
 * for tiles without intersections. Returns the number of real (non-padding) entries.
 */
int orc_sort_intersects(int n, int capacity, const float *xys, const int *radii, const int *cum, int tiles_x, int tiles_y,
                        int *gaussian_ids_sorted, int *tile_bins) {
    const int num_tiles = tiles_x * tiles_y;
    memset(tile_bins, 0, sizeof(int) * 2 * (size_t)num_tiles);
    if (capacity <= 0) return 0;
    keyval *kv = (keyval *)malloc(sizeof(keyval) * (size_t)capacity);
    for (int i = 0; i < capacity; ++i) {
        kv[i].key = (uint32_t)num_tiles;
        kv[i].val = 0;
        kv[i].pos = i;
    }
    int real = 0;
    if (n > 0) {
        int total = cum[n - 1];
        int limit = total < capacity ? total : capacity;
        for (int idx = 0; idx < limit; ++idx) {
            int lo = 0, hi = n - 1;
            while (lo < hi) {
                int mid = (lo + hi) / 2;
                if (cum[mid] > idx)
                    hi = mid;
                else
                    lo = mid + 1;
            }
            int local = idx - (lo == 0 ? 0 : cum[lo - 1]);
            int x0, y0, x1, y1;
            tile_bbox(xys[2 * lo], xys[2 * lo + 1], (float)radii[lo], tiles_x, tiles_y, &x0, &y0, &x1, &y1);
            int width = x1 - x0;
            if (width <= 0) continue; /* inconsistent inputs; the reference would divide by zero */
            kv[idx].key = (uint32_t)((y0 + local / width) * tiles_x + x0 + local % width);
            kv[idx].val = lo;
        }
        real = limit > 0 ? limit : 0;
    }
    qsort(kv, (size_t)capacity, sizeof(keyval), keyval_cmp);
    for (int i = 0; i < capacity; ++i) gaussian_ids_sorted[i] = kv[i].val;
    for (int i = 0; i < capacity; ++i) {
        uint32_t t = kv[i].key;
        if (t >= (uint32_t)num_tiles) continue;
        if (i == 0 || kv[i - 1].key != t) tile_bins[2 * t] = i;
        if (i == capacity - 1 || kv[i + 1].key != t) tile_bins[2 * t + 1] = i + 1;
    }
    free(kv);
    return real;
}

/* __expf(-sigma) of the reference: IEEE expf, with results below FLT_MIN flushed to zero as the fast-math (ftz) intrinsic does */
static float alpha_of(float sigma) {
    float a = expf(-sigma);
    return a < FLT_MIN ? 0.f : a;
}

static float sigma_of(const float *xy, const float *conic, float px, float py) {
    float dx = xy[0] - px, dy = xy[1] - py;
    return 0.5f * (conic[0] * dx * dx + conic[2] * dy * dy) + conic[1] * dx * dy;
}

/*
 * Top-K normalized forward: nd_rasterize_forward_topk_norm (forward.cu:223-375). Per pixel (integer coordinates px = j, py = i), walk the
 * tile's list in order; skip sigma < 0, NaN or Inf; alpha enters if alpha > the cached minimum (-1 while slots are free), into the next
 * free slot, else into the first slot holding the strict minimum, after which the minimum is rescanned. The output normalizes in double
 * (sum + 1e-4, a double literal) and accumulates channels over slots in slot order. Image [C, H, W], pixel_topk [H, W, 10] (-1 empty).
 */
typedef struct {
    int tiles_x, img_h, img_w, channels;
    const int *gaussian_ids_sorted, *tile_bins;
    const float *xys, *conics, *colors;
    float *out_img;
    int *pixel_topk;
} fwd_ctx;

static void raster_fwd_tiles(void *arg, int tile_begin, int tile_end) {
    const fwd_ctx *x = (const fwd_ctx *)arg;
    const int img_h = x->img_h, img_w = x->img_w, channels = x->channels, num_pixels = img_h * img_w;
    for (int tile = tile_begin; tile < tile_end; ++tile) {
        const int tx = tile % x->tiles_x, ty = tile / x->tiles_x;
        const int start = x->tile_bins[2 * tile], end = x->tile_bins[2 * tile + 1];
        for (int ly = 0; ly < ORC_TILE; ++ly) {
            for (int lx = 0; lx < ORC_TILE; ++lx) {
                const int i = ty * ORC_TILE + ly, j = tx * ORC_TILE + lx;
                if (i >= img_h || j >= img_w) continue;
                const float px = (float)j, py = (float)i;
                int ids[ORC_TOPK];
                float vals[ORC_TOPK];
                for (int k = 0; k < ORC_TOPK; ++k) {
                    ids[k] = -1;
                    vals[k] = 0.f;
                }
                int filled = 0, min_slot = 0;
                float min_val = -1.f;
                for (int idx = start; idx < end; ++idx) {
                    const int g = x->gaussian_ids_sorted[idx];
                    const float sigma = sigma_of(&x->xys[2 * g], &x->conics[3 * g], px, py);
                    if (sigma < 0.f || isnan(sigma) || isinf(sigma)) continue;
                    const float alpha = alpha_of(sigma);
                    if (!(alpha > min_val)) continue;
                    const int slot = filled < ORC_TOPK ? filled : min_slot;
                    ids[slot] = g;
                    vals[slot] = alpha;
                    if (filled < ORC_TOPK) ++filled;
                    if (filled == ORC_TOPK) {
                        min_slot = 0;
                        min_val = vals[0];
                        for (int k = 1; k < ORC_TOPK; ++k)
                            if (vals[k] < min_val) {
                                min_slot = k;
                                min_val = vals[k];
                            }
                    }
                }
                float sum = 0.f;
                for (int k = 0; k < ORC_TOPK; ++k)
                    if (ids[k] >= 0) sum += vals[k];
                float out[ORC_MAX_CHANNELS] = {0.f};
                for (int k = 0; k < ORC_TOPK; ++k) {
                    if (ids[k] < 0) continue;
                    const float vis = (float)((double)vals[k] / ((double)sum + ORC_EPS));
                    for (int c = 0; c < channels; ++c) out[c] += x->colors[ids[k] * channels + c] * vis;
                }
                const int pix = i * img_w + j;
                for (int c = 0; c < channels; ++c) x->out_img[(size_t)c * num_pixels + pix] = out[c];
                for (int k = 0; k < ORC_TOPK; ++k) x->pixel_topk[(size_t)pix * ORC_TOPK + k] = ids[k];
            }
        }
    }
}

void orc_raster_fwd(int tiles_x, int tiles_y, int img_h, int img_w, int channels, const int *gaussian_ids_sorted, const int *tile_bins,
                    const float *xys, const float *conics, const float *colors, float *out_img, int *pixel_topk) {
    fwd_ctx ctx = {tiles_x, img_h, img_w, channels, gaussian_ids_sorted, tile_bins, xys, conics, colors, out_img, pixel_topk};
    parallel_for(tiles_x * tiles_y, 16, raster_fwd_tiles, &ctx);
}

/*
 * Top-K normalized backward: the per-pixel algebra of nd_rasterize_backward_topk_norm_kernel (backward.cu:219-265) and the per-Gaussian
 * values it adds (backward.cu:292-306), summed here per Gaussian in double in pixel order (the reference adds them with unordered float
 * atomics). With D = 1e-4 + sum_k d_k, s_k = f_k . v_out, dL/dd_k = s_k / D - sum_j d_j s_j / D^2, v_sigma_k = -d_k dL/dd_k:
 * v_conic += (v_sigma dx^2 / 2, v_sigma dx dy, v_sigma dy^2 / 2), v_xy += v_sigma (a dx + b dy, b dx + c dy), v_color += d_k / D v_out.
 * Outputs v_xy [N, 2], v_conic [N, 3], v_colors [N, C] are overwritten.
 */
typedef struct {
    int img_h, img_w, channels, n, parts;
    const float *xys, *conics, *colors, *v_output;
    const int *pixel_topk;
    double *acc; /* parts x n x (5 + C) */
    int absolute; /* sum the terms' magnitudes instead (orc_raster_bwd_abs) */
} bwd_ctx;

static void raster_bwd_part(void *arg, int part_begin, int part_end) {
    const bwd_ctx *x = (const bwd_ctx *)arg;
    const int num_pixels = x->img_h * x->img_w, channels = x->channels, nv = 5 + channels;
    for (int part = part_begin; part < part_end; ++part) {
        double *acc = x->acc + (size_t)part * x->n * nv;
        const int p0 = (int)((int64_t)num_pixels * part / x->parts), p1 = (int)((int64_t)num_pixels * (part + 1) / x->parts);
        for (int pix = p0; pix < p1; ++pix) {
            const float px = (float)(pix % x->img_w), py = (float)(pix / x->img_w);
            float v_out[ORC_MAX_CHANNELS];
            for (int c = 0; c < channels; ++c) v_out[c] = x->v_output[(size_t)c * num_pixels + pix];
            int ids[ORC_TOPK];
            float d[ORC_TOPK];
            float denom = (float)ORC_EPS;
            for (int k = 0; k < ORC_TOPK; ++k) {
                ids[k] = x->pixel_topk[(size_t)pix * ORC_TOPK + k];
                d[k] = 0.f;
                if (ids[k] < 0) continue;
                d[k] = alpha_of(sigma_of(&x->xys[2 * ids[k]], &x->conics[3 * ids[k]], px, py));
                denom += d[k];
            }
            float s[ORC_TOPK];
            float shared = 0.f;
            for (int k = 0; k < ORC_TOPK; ++k) {
                s[k] = 0.f;
                if (ids[k] < 0) continue;
                for (int c = 0; c < channels; ++c) s[k] += x->colors[ids[k] * channels + c] * v_out[c];
                shared += -d[k] / (denom * denom) * s[k];
            }
            for (int k = 0; k < ORC_TOPK; ++k) {
                if (ids[k] < 0) continue;
                const int g = ids[k];
                const float w = d[k] / denom;
                const float vs = -d[k] * (s[k] / denom + shared);
                const float dx = x->xys[2 * g] - px, dy = x->xys[2 * g + 1] - py;
                const float a = x->conics[3 * g], b = x->conics[3 * g + 1], c2 = x->conics[3 * g + 2];
                double *o = &acc[(size_t)g * nv];
                if (x->absolute) {
                    o[0] += fabs(0.5f * vs * dx * dx);
                    o[1] += fabs(vs * dx * dy);
                    o[2] += fabs(0.5f * vs * dy * dy);
                    o[3] += fabs(vs * (a * dx + b * dy));
                    o[4] += fabs(vs * (b * dx + c2 * dy));
                    for (int c = 0; c < channels; ++c) o[5 + c] += fabs(w * v_out[c]);
                    continue;
                }
                o[0] += 0.5f * vs * dx * dx;
                o[1] += vs * dx * dy;
                o[2] += 0.5f * vs * dy * dy;
                o[3] += vs * (a * dx + b * dy);
                o[4] += vs * (b * dx + c2 * dy);
                for (int c = 0; c < channels; ++c) o[5 + c] += w * v_out[c];
            }
        }
    }
}

static void raster_bwd_sums(int img_h, int img_w, int channels, int n, const float *xys, const float *conics, const float *colors,
                            const float *v_output, const int *pixel_topk, float *v_xy, float *v_conic, float *v_colors, int absolute) {
    const int nv = 5 + channels;
    /* static pixel ranges per part, each with its own accumulator, summed in part order: deterministic for a given thread count */
    const int parts = g_threads;
    double *acc = (double *)calloc((size_t)parts * n * nv, sizeof(double));
    bwd_ctx ctx = {img_h, img_w, channels, n, parts, xys, conics, colors, v_output, pixel_topk, acc, absolute};
    parallel_for(parts, 1, raster_bwd_part, &ctx);
    for (int g = 0; g < n; ++g) {
        double o[5 + ORC_MAX_CHANNELS] = {0.0};
        for (int part = 0; part < parts; ++part)
            for (int v = 0; v < nv; ++v) o[v] += acc[((size_t)part * n + g) * nv + v];
        v_conic[3 * g] = (float)o[0];
        v_conic[3 * g + 1] = (float)o[1];
        v_conic[3 * g + 2] = (float)o[2];
        v_xy[2 * g] = (float)o[3];
        v_xy[2 * g + 1] = (float)o[4];
        for (int c = 0; c < channels; ++c) v_colors[(size_t)g * channels + c] = (float)o[5 + c];
    }
    free(acc);
}

void orc_raster_bwd(int img_h, int img_w, int channels, int n, const float *xys, const float *conics, const float *colors,
                    const float *v_output, const int *pixel_topk, float *v_xy, float *v_conic, float *v_colors) {
    raster_bwd_sums(img_h, img_w, channels, n, xys, conics, colors, v_output, pixel_topk, v_xy, v_conic, v_colors, 0);
}

/*
 * The magnitudes of the same per-pixel terms summed per Gaussian: sum |term| for each value of v_xy, v_conic, v_colors. Two float
 * summations of one gradient in different orders differ by up to a small multiple of the unit roundoff times this sum, however much the
 * terms cancel; the tests use it as the scale of that rounding.
 */
void orc_raster_bwd_abs(int img_h, int img_w, int channels, int n, const float *xys, const float *conics, const float *colors,
                        const float *v_output, const int *pixel_topk, float *v_xy, float *v_conic, float *v_colors) {
    raster_bwd_sums(img_h, img_w, channels, n, xys, conics, colors, v_output, pixel_topk, v_xy, v_conic, v_colors, 1);
}

/*
 * Leave-one-out loss increase: topk_norm_loo_loss_increase (forward.cu:667-738), restated literally in float per pixel: with the top-K
 * weights w = exp(-sigma), S_w = sum_k w_k and S_f = sum_k w_k f_k in slot order, the pixel's error sum_c |S_f / (S_w + eps) - t| (or its
 * square), and for each top-K Gaussian the error of (S_f - w_k f_k) / (S_w - w_k + eps); their difference is added to the Gaussian (here
 * summed in double; the reference uses float atomics). Used by pruning rounds, not by the training step.
 */
void orc_loo_loss_increase(int img_h, int img_w, int channels, int n, const float *xys, const float *conics, const float *colors,
                           const int *pixel_topk, const float *targets, int squared, float eps, float *loss_increase) {
    const int num_pixels = img_h * img_w;
    double *acc = (double *)calloc((size_t)n, sizeof(double));
    for (int pix = 0; pix < num_pixels; ++pix) {
        const float px = (float)(pix % img_w), py = (float)(pix / img_w);
        int ids[ORC_TOPK];
        float w[ORC_TOPK], sum_w = 0.f, sum_f[ORC_MAX_CHANNELS], target[ORC_MAX_CHANNELS];
        for (int c = 0; c < channels; ++c) {
            sum_f[c] = 0.f;
            target[c] = targets[(size_t)c * num_pixels + pix];
        }
        for (int k = 0; k < ORC_TOPK; ++k) {
            ids[k] = pixel_topk[(size_t)pix * ORC_TOPK + k];
            w[k] = 0.f;
            if (ids[k] < 0) continue;
            w[k] = alpha_of(sigma_of(&xys[2 * ids[k]], &conics[3 * ids[k]], px, py));
            sum_w += w[k];
            for (int c = 0; c < channels; ++c) sum_f[c] += w[k] * colors[ids[k] * channels + c];
        }
        float error = 0.f;
        for (int c = 0; c < channels; ++c) {
            const float diff = sum_f[c] / (sum_w + eps) - target[c];
            error += squared ? diff * diff : fabsf(diff);
        }
        for (int k = 0; k < ORC_TOPK; ++k) {
            const int g = ids[k];
            if (g < 0) continue;
            const float inv = 1.f / (sum_w - w[k] + eps);
            float loo = 0.f;
            for (int c = 0; c < channels; ++c) {
                const float diff = (sum_f[c] - w[k] * colors[g * channels + c]) * inv - target[c];
                loo += squared ? diff * diff : fabsf(diff);
            }
            acc[g] += loo - error;
        }
    }
    for (int g = 0; g < n; ++g) loss_increase[g] = (float)acc[g];
    free(acc);
}
