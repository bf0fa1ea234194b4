/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU restatement of gpu.RunCPU's
 * results for simtgo's hot-path kernels. See oracle.h for who may use it.
 *
 * Each function follows the Go kernel body it names, under the grid rules of
 * gpu/gpu.go:244-431: a thread acts only if its global index is below
 * grid*block; blocks are independent and may run in any order, so they are
 * handed to a pool of worker threads (gpu/gpu.go:319-356).
 *
 * Compile with -ffp-contract=off (oracle/Makefile): amd64 Go rounds every
 * float32 operation on its own (NUMERICS.md:103-118).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Status codes shared with include/simtgo_b200.h. */
#define E_NULL (-1)
#define E_LENGTH (-2)
#define E_BLOCK (-3)
#define E_LAUNCH (-5)
#define E_TAPS (-6)
#define E_GRAPH (-7)
#define E_ARG (-11)

static int g_threads = 1;
void oracle_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int oracle_get_threads(void) { return g_threads; }

/* ---- a block-parallel loop: runCPU's worker pool ----------------------- */
typedef void (*range_fn)(int64_t lo, int64_t hi, void* ctx);
typedef struct {
    range_fn fn;
    void* ctx;
    int64_t lo, hi;
} par_job;

static void* par_worker(void* p) {
    par_job* j = (par_job*)p;
    j->fn(j->lo, j->hi, j->ctx);
    return NULL;
}

static void par_for(int64_t n, range_fn fn, void* ctx) {
    int nt = g_threads;
    if (n <= 0) return;
    if (nt > n) nt = (int)n;
    if (nt <= 1) {
        fn(0, n, ctx);
        return;
    }
    pthread_t th[256];
    par_job jobs[256];
    memset(jobs, 0, sizeof jobs);
    if (nt > 256) nt = 256;
    int64_t per = (n + nt - 1) / nt;
    int started = 0;
    for (int t = 0; t < nt; t++) {
        int64_t lo = t * per, hi = lo + per < n ? lo + per : n;
        if (lo >= hi) break;
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].lo = lo;
        jobs[t].hi = hi;
        if (t == 0) continue; /* run the first range on this thread */
        pthread_create(&th[t], NULL, par_worker, &jobs[t]);
        started = t;
    }
    fn(jobs[0].lo, jobs[0].hi, ctx);
    for (int t = 1; t <= started; t++) pthread_join(th[t], NULL);
}

static int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

/* The global indices a 1-D launch covers, and whether the launch is valid
 * for the device (gpu.RunCPU itself just returns for an empty grid). */
static int launch_extent(int64_t grid, int64_t block, int64_t* threads) {
    if (grid <= 0 || block <= 0 || block > 1024) return E_LAUNCH;
    *threads = grid * block;
    return 0;
}

/* ---- gpu.Hypot: math.Hypot on float64, rounded to float32 --------------
 * Go's math.Hypot (and its amd64 assembly, the same steps): absolute values;
 * +Inf if either is infinite; NaN if either is NaN; then
 * max * Sqrt(1 + (min/max)^2), 0 when both are zero. */
static double go_hypot(double p, double q) {
    p = fabs(p);
    q = fabs(q);
    if (isinf(p) || isinf(q)) return INFINITY;
    if (isnan(p) || isnan(q)) return NAN;
    if (p < q) {
        double t = p;
        p = q;
        q = t;
    }
    if (p == 0) return 0;
    q = q / p;
    return p * sqrt(1 + q * q);
}
float oracle_hypot(float x, float y) { return (float)go_hypot((double)x, (double)y); }

/* ---- elementwise kernels ------------------------------------------------ */
typedef struct {
    float* out;
    const float *a, *b;
    float k;
} ew_ctx;

static void vecadd_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = c->a[i] + c->b[i];
}
/* kernels/kernels.go:12-17 */
int oracle_vecadd(float* c, int32_t c_len, const float* a, int32_t a_len, const float* b,
                  int32_t b_len, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(c_len, nt);
    if (m <= 0) return 0;
    if (a_len < m || b_len < m) return E_LENGTH;
    ew_ctx ctx = {c, a, b, 0};
    par_for(m, vecadd_range, &ctx);
    return 0;
}

static void scale_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = c->k * c->a[i];
}
/* kernels/kernels.go:29-34 */
int oracle_scale(float* y, int32_t y_len, const float* x, int32_t x_len, float k, int64_t grid,
                 int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(y_len, nt);
    if (m <= 0) return 0;
    if (x_len < m) return E_LENGTH;
    ew_ctx ctx = {y, x, NULL, k};
    par_for(m, scale_range, &ctx);
    return 0;
}

static void magnitude_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = oracle_hypot(c->a[i], c->b[i]);
}
/* kernels/kernels.go:21-26 with gpu.Hypot (gpu/math.go:17) */
int oracle_magnitude(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                     const float* im, int32_t im_len, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(mag_len, nt);
    if (m <= 0) return 0;
    if (re_len < m || im_len < m) return E_LENGTH;
    ew_ctx ctx = {mag, re, im, 0};
    par_for(m, magnitude_range, &ctx);
    return 0;
}

/* gpu.Sqrt (gpu/math.go:11): the float64 square root rounded to float32,
 * which equals the correctly rounded float32 square root. */
static float go_sqrt32(float x) { return (float)sqrt((double)x); }

static float magfast_one(float r, float m, float scale) {
    float rr = r * r;
    float mm = m * m;
    float s = rr + mm;
    return go_sqrt32(s) / scale;
}
static void magfast_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = magfast_one(c->a[i], c->b[i], c->k);
}
/* kernels/magnitudefast.go:20-26 */
int oracle_magnitudefast(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                         const float* im, int32_t im_len, float scale, int64_t grid,
                         int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(mag_len, nt);
    if (m <= 0) return 0;
    if (re_len < m || im_len < m) return E_LENGTH;
    ew_ctx ctx = {mag, re, im, scale};
    par_for(m, magfast_range, &ctx);
    return 0;
}

static void magfast_il_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = magfast_one(c->a[2 * i], c->a[2 * i + 1], c->k);
}
int oracle_magnitudefast_interleaved(float* mag, int32_t mag_len, const float* z, int32_t z_len,
                                     float scale, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(mag_len, nt);
    if (m <= 0) return 0;
    if ((int64_t)z_len < 2 * m) return E_LENGTH;
    ew_ctx ctx = {mag, z, NULL, scale};
    par_for(m, magfast_il_range, &ctx);
    return 0;
}

/* kernels/softclip.go:11-23 */
static float softclip_one(float v, float threshold) {
    float a = fabsf(v);
    if (a <= threshold) return v;
    float over = a - threshold;
    float shaped = threshold + over / (1.0f + over);
    if (v < 0) return -shaped;
    return shaped;
}
static void softclip_range(int64_t lo, int64_t hi, void* p) {
    ew_ctx* c = (ew_ctx*)p;
    for (int64_t i = lo; i < hi; i++) c->out[i] = softclip_one(c->a[i], c->k);
}
/* kernels/softclip.go:25-30 */
int oracle_softclip(float* y, int32_t y_len, const float* x, int32_t x_len, float threshold,
                    int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(y_len, nt);
    if (m <= 0) return 0;
    if (x_len < m) return E_LENGTH;
    ew_ctx ctx = {y, x, NULL, threshold};
    par_for(m, softclip_range, &ctx);
    return 0;
}

typedef struct {
    float* out;
    const float* x;
    const float* edges;
    int32_t n_edges;
    float bias;
} classify_ctx;
static void classify_range(int64_t lo, int64_t hi, void* p) {
    classify_ctx* c = (classify_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        float v = fabsf(c->x[i]);
        /* The grouped scan with a labelled break (classify.go:23-34) finds
         * the first edge v does not exceed. */
        int32_t band = c->n_edges;
        for (int32_t j = 0; j < c->n_edges; j++) {
            if (v <= c->edges[j]) {
                band = j;
                break;
            }
        }
        float gain;
        switch (band) {
            case 0: gain = 0.25f; break;
            case 1:
            case 2: gain = 0.5f; break;
            case 3: gain = 0.75f; break;
            default: gain = 1.0f; break;
        }
        float gv = gain * v;
        float b = c->bias * 0.001f;
        c->out[i] = gv + b;
    }
}
/* kernels/classify.go:14-56 */
int oracle_classify(float* out, int32_t out_len, const float* x, int32_t x_len,
                    const float* edges, int32_t edges_len, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(out_len, nt);
    if (m <= 0) return 0;
    if (x_len < m) return E_LENGTH;
    if (edges_len < 0) edges_len = 0;
    float bias = 0;
    for (int32_t j = 0; j < edges_len; j++) bias += edges[j];
    classify_ctx ctx = {out, x, edges, edges_len, bias};
    par_for(m, classify_range, &ctx);
    return 0;
}

typedef struct {
    float* y;
    const float* x;
    int32_t x_len;
    const oracle_band* bands;
    int32_t n_bands;
    oracle_shape cfg;
} bandgain_ctx;
static void bandgain_range(int64_t lo, int64_t hi, void* p) {
    bandgain_ctx* c = (bandgain_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        float v = c->x[i];
        float gain = c->cfg.floor_gain;
        for (int32_t b = 0; b < c->n_bands; b++) {
            if (v <= c->bands[b].upper) {
                gain = c->bands[b].gain;
                break;
            }
        }
        float taps[4] = {0, 0, 0, 0};
        for (int j = 0; j < 4; j++) {
            int64_t k = i + j - 2;
            if (k >= 0 && k < c->x_len) taps[j] = c->x[k];
        }
        float sum = 0;
        for (int j = 0; j < 4; j++) sum += taps[j];
        double acc = (double)sum / 4.0;
        acc = acc * (double)gain;
        acc = acc + c->cfg.bias;
        c->y[i] = (float)acc * (float)c->cfg.count;
    }
}
/* kernels/bandgain.go:42-76 */
int oracle_bandgain(float* y, int32_t y_len, const float* x, int32_t x_len,
                    const oracle_band* bands, int32_t bands_len, const oracle_shape* cfg,
                    int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    if (!cfg) return E_NULL;
    int64_t m = min64(y_len, nt);
    if (m <= 0) return 0;
    if (x_len < m) return E_LENGTH;
    if (bands_len < 0) bands_len = 0;
    bandgain_ctx ctx = {y, x, x_len, bands, bands_len, *cfg};
    par_for(m, bandgain_range, &ctx);
    return 0;
}

/* Go's float32 -> int32 conversion on amd64 (CVTTSS2SL): truncation, and
 * 0x80000000 for NaN or a value out of range. */
static int32_t go_f32_to_i32(float f) {
    if (f >= -2147483648.0f && f < 2147483648.0f) return (int32_t)f;
    return INT32_MIN;
}

typedef struct {
    int32_t* code;
    int64_t* energy;
    uint8_t* clipped;
    const float* x;
    float step;
    uint32_t seed;
} quantize_ctx;
static void quantize_range(int64_t lo, int64_t hi, void* p) {
    quantize_ctx* c = (quantize_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        uint32_t h = c->seed ^ (uint32_t)i;
        h = h * 2654435761u + 1u;
        h ^= h >> 15;
        float jitter = (float)(int32_t)(h % 1024u) / 1024.0f - 0.5f;
        float q0 = c->x[i] / c->step;
        q0 = q0 + jitter;
        int32_t q = go_f32_to_i32(q0);
        uint8_t cl;
        if (q > 127) {
            q = 127;
            cl = 1;
        } else if (q < -128) {
            q = -128;
            cl = 1;
        } else {
            cl = 0;
        }
        c->clipped[i] = cl;
        c->code[i] = q;
        c->energy[i] = (int64_t)q * (int64_t)q;
    }
}
/* kernels/quantize.go:16-45 */
int oracle_quantize(int32_t* code, int32_t code_len, int64_t* energy, int32_t energy_len,
                    uint8_t* clipped, int32_t clipped_len, const float* x, int32_t x_len,
                    float step, uint32_t seed, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(code_len, nt);
    if (m <= 0) return 0;
    if (x_len < m || energy_len < m || clipped_len < m) return E_LENGTH;
    quantize_ctx ctx = {code, energy, clipped, x, step, seed};
    par_for(m, quantize_range, &ctx);
    return 0;
}

typedef struct {
    uint8_t* out;
    const uint8_t* rgb;
    int64_t rgb_len;
} gray_ctx;
static void gray_range(int64_t lo, int64_t hi, void* p) {
    gray_ctx* c = (gray_ctx*)p;
    for (int64_t i = lo; i < hi; i++) {
        int64_t j = i * 3;
        if (j + 2 >= c->rgb_len) continue;
        int32_t r = c->rgb[j], g = c->rgb[j + 1], b = c->rgb[j + 2];
        int32_t y = (77 * r + 150 * g + 29 * b + 128) >> 8;
        c->out[i] = (uint8_t)y;
    }
}
/* kernels/gray.go:34-55 */
int oracle_gray(uint8_t* out, int32_t out_len, const uint8_t* rgb, int32_t rgb_len, int64_t grid,
                int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(out_len, nt);
    if (m <= 0) return 0;
    gray_ctx ctx = {out, rgb, rgb_len};
    par_for(m, gray_range, &ctx);
    return 0;
}

/* ---- histogram: one privatised tile per block -------------------------- */
typedef struct {
    int32_t* bins;
    int32_t n_bins;
    const int32_t* x;
    int64_t m;
    int64_t block;
    pthread_mutex_t mu; /* gpu.AtomicAddI32's lock (gpu/atomic.go:42) */
} hist_ctx;
static void hist_range(int64_t lo, int64_t hi, void* p) {
    hist_ctx* c = (hist_ctx*)p;
    int32_t tile[256];
    int32_t acc[256];
    memset(acc, 0, sizeof acc);
    for (int64_t blk = lo; blk < hi; blk++) {
        memset(tile, 0, sizeof tile);
        int64_t i0 = blk * c->block, i1 = min64(i0 + c->block, c->m);
        for (int64_t i = i0; i < i1; i++) {
            int32_t v = c->x[i];
            if (v >= 0 && v < 256) tile[v]++;
        }
        for (int k = 0; k < 256; k++) acc[k] += tile[k];
    }
    pthread_mutex_lock(&c->mu);
    for (int k = 0; k < 256 && k < c->n_bins; k++)
        c->bins[k] = (int32_t)((uint32_t)c->bins[k] + (uint32_t)acc[k]);
    pthread_mutex_unlock(&c->mu);
}
/* kernels/histogram.go:23-50 */
int oracle_histogram(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                     int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    int64_t m = min64(x_len, nt);
    if (m <= 0) return 0;
    hist_ctx ctx;
    ctx.bins = bins;
    ctx.n_bins = bins_len;
    ctx.x = x;
    ctx.m = m;
    ctx.block = block;
    pthread_mutex_init(&ctx.mu, NULL);
    par_for((m + block - 1) / block, hist_range, &ctx);
    pthread_mutex_destroy(&ctx.mu);
    return 0;
}

/* The launch-sized tile (simt Kernel.LaunchShared, simt/kernel.go:444-481)
 * on the DynProbe body (simt/shared_parity_cuda_test.go:117-138): each block
 * zeroes a tile of tile_len int32, counts its samples x[i] in [0, tile_len)
 * with gpu.AtomicAddI32, then adds every non-zero tile[k], k < bins_len,
 * into bins[k]. Integer sums are order-free, so one pass per block range is
 * the same result. */
typedef struct {
    int32_t* bins;
    int32_t n_bins, tile;
    const int32_t* x;
    int64_t m, block;
    pthread_mutex_t mu;
} hdyn_ctx;
static void hdyn_range(int64_t lo, int64_t hi, void* p) {
    hdyn_ctx* c = (hdyn_ctx*)p;
    int32_t* acc = (int32_t*)calloc((size_t)(c->tile > 0 ? c->tile : 1), sizeof(int32_t));
    for (int64_t blk = lo; blk < hi; blk++) {
        int64_t i0 = blk * c->block, i1 = min64(i0 + c->block, c->m);
        for (int64_t i = i0; i < i1; i++) {
            int32_t v = c->x[i];
            if (v >= 0 && v < c->tile) acc[v]++;
        }
    }
    pthread_mutex_lock(&c->mu);
    for (int32_t k = 0; k < c->tile && k < c->n_bins; k++)
        c->bins[k] = (int32_t)((uint32_t)c->bins[k] + (uint32_t)acc[k]);
    pthread_mutex_unlock(&c->mu);
    free(acc);
}
int oracle_histogram_dyn(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                         int32_t tile_len, int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    if (tile_len < 0) return E_ARG;
    int64_t m = min64(x_len, nt);
    if (m <= 0 || tile_len == 0) return 0;
    hdyn_ctx ctx;
    ctx.bins = bins;
    ctx.n_bins = bins_len;
    ctx.tile = tile_len;
    ctx.x = x;
    ctx.m = m;
    ctx.block = block;
    pthread_mutex_init(&ctx.mu, NULL);
    par_for((m + block - 1) / block, hdyn_range, &ctx);
    pthread_mutex_destroy(&ctx.mu);
    return 0;
}

int oracle_histogram_shard(int32_t* bins, int32_t bins_len, const int32_t* x, int64_t x_len) {
    if (x_len <= 0) return 0;
    hist_ctx ctx;
    ctx.bins = bins;
    ctx.n_bins = bins_len;
    ctx.x = x;
    ctx.m = x_len;
    ctx.block = 1 << 16;
    pthread_mutex_init(&ctx.mu, NULL);
    par_for((x_len + ctx.block - 1) / ctx.block, hist_range, &ctx);
    pthread_mutex_destroy(&ctx.mu);
    return 0;
}

/* ---- transpose ---------------------------------------------------------- */
typedef struct {
    float* out;
    const float* in;
    int64_t w, h, xcov, ycov;
} tr_ctx;
static void transpose_range(int64_t lo, int64_t hi, void* p) {
    tr_ctx* c = (tr_ctx*)p;
    for (int64_t ox = lo; ox < hi; ox++) /* ox = source row */
        for (int64_t oy = 0; oy < c->xcov; oy++) c->out[oy * c->h + ox] = c->in[ox * c->w + oy];
}
/* kernels/transpose.go:15-38. A block (bx, by) stages in[y][x] for x < w,
 * y < h of its 16x16 tile and writes out[oy*h + ox] = in[ox*w + oy] for
 * ox < h, oy < w of the swapped tile: the covered rectangle transposed. */
int oracle_transpose(float* out, int32_t out_len, const float* in, int32_t in_len, int32_t w,
                     int32_t h, int64_t grid_x, int64_t grid_y, int64_t block_x,
                     int64_t block_y) {
    if (grid_x <= 0 || grid_y <= 0 || block_x <= 0 || block_y <= 0) return E_LAUNCH;
    if (block_x * block_y != 256) return E_BLOCK;
    if (block_x != 16 || block_y != 16) return E_BLOCK;
    int64_t xcov = min64(w, grid_x * 16), ycov = min64(h, grid_y * 16);
    if (xcov <= 0 || ycov <= 0) return 0;
    if ((ycov - 1) * (int64_t)w + (xcov - 1) >= in_len) return E_LENGTH;
    if ((xcov - 1) * (int64_t)h + (ycov - 1) >= out_len) return E_LENGTH;
    tr_ctx ctx = {out, in, w, h, xcov, ycov};
    par_for(ycov, transpose_range, &ctx);
    return 0;
}

/* ---- warp reduction ----------------------------------------------------- */
typedef struct {
    float* out;
    int64_t n_out;
    const float* x;
    int64_t x_len;
} wr_ctx;
static void warpreduce_range(int64_t lo, int64_t hi, void* p) {
    wr_ctx* c = (wr_ctx*)p;
    for (int64_t w = lo; w < hi; w++) {
        float v[32], nv[32];
        for (int l = 0; l < 32; l++) {
            int64_t i = w * 32 + l;
            v[l] = i < c->x_len ? c->x[i] : 0.0f;
        }
        /* gpu.ShuffleDownF32 (gpu/warp.go:127): a lane past the end of the
         * warp gets its own value back. */
        for (int off = 16; off > 0; off /= 2) {
            for (int l = 0; l < 32; l++) nv[l] = v[l] + (l + off < 32 ? v[l + off] : v[l]);
            memcpy(v, nv, sizeof v);
        }
        c->out[w] = v[0];
    }
}
/* kernels/warpreduce.go:21-43 */
int oracle_warpreducesum(float* out, int32_t out_len, const float* x, int32_t x_len,
                         int64_t grid, int64_t block) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    if (block != 128) return E_BLOCK;
    int64_t warps = min64(out_len, nt / 32);
    if (warps <= 0) return 0;
    wr_ctx ctx = {out, warps, x, x_len < 0 ? 0 : x_len};
    par_for(warps, warpreduce_range, &ctx);
    return 0;
}

/* ---- FIR ---------------------------------------------------------------- */
typedef struct {
    float* y;
    int64_t y_len;
    const float* x;
    int64_t x_len;
    int64_t halo;
    const float* h;
    int32_t taps;
    int fused;
} fir_ctx;
#define FIR_CHUNK 256
/* Outputs [lo, hi) in chunks of 256 (one FIRBlock), each staged as the
 * reference's tile: x at (j - k) for k < taps, zero outside [0, x_len). The
 * loop over t is innermost so the compiler can vectorise across outputs while
 * each output keeps its own k order. */
static void fir_range(int64_t lo_chunk, int64_t hi_chunk, void* p) {
    fir_ctx* c = (fir_ctx*)p;
    int32_t taps = c->taps;
    float tile[FIR_CHUNK + 1024 + 1];
    float acc[FIR_CHUNK];
    for (int64_t ch = lo_chunk; ch < hi_chunk; ch++) {
        int64_t base = ch * FIR_CHUNK;
        int64_t cnt = min64(FIR_CHUNK, c->y_len - base);
        int32_t span = FIR_CHUNK + (taps > 0 ? taps - 1 : 0);
        for (int32_t k = 0; k < span; k++) {
            int64_t src = base + c->halo + k - (taps > 0 ? taps - 1 : 0);
            tile[k] = (src >= 0 && src < c->x_len) ? c->x[src] : 0.0f;
        }
        for (int t = 0; t < FIR_CHUNK; t++) acc[t] = 0.0f;
        for (int32_t k = 0; k < taps; k++) {
            const float hk = c->h[k];
            const float* s = tile + (taps - 1 - k);
            if (c->fused) {
                for (int t = 0; t < FIR_CHUNK; t++) acc[t] = fmaf(hk, s[t], acc[t]);
            } else {
                for (int t = 0; t < FIR_CHUNK; t++) {
                    float prod = hk * s[t];
                    acc[t] = acc[t] + prod;
                }
            }
        }
        memcpy(c->y + base, acc, (size_t)cnt * sizeof(float));
    }
}

static int fir_common(float* y, int32_t y_len, const float* x, int32_t x_len, const float* h,
                      int32_t h_len, int64_t grid, int64_t block, int fused) {
    int64_t nt;
    int rc = launch_extent(grid, block, &nt);
    if (rc) return rc;
    if (block != 256) return E_BLOCK;
    /* The staged tile is FIRBlock+FIRMaxTaps = 320 samples (fir.go:24);
     * gpu.RunCPU panics on a tap count whose halo does not fit. */
    if (h_len < 0 || h_len > 65) return E_TAPS;
    int64_t m = min64(y_len, nt);
    if (m <= 0) return 0;
    fir_ctx ctx = {y, m, x, x_len < 0 ? 0 : x_len, 0, h, h_len, fused};
    par_for((m + FIR_CHUNK - 1) / FIR_CHUNK, fir_range, &ctx);
    return 0;
}
/* kernels/fir.go:17-46 as gpu.RunCPU runs it */
int oracle_fir(float* y, int32_t y_len, const float* x, int32_t x_len, const float* h,
               int32_t h_len, int64_t grid, int64_t block) {
    return fir_common(y, y_len, x, x_len, h, h_len, grid, block, 0);
}
/* kernels/prebuilt/FIR.cu:22-27 as nvcc contracts it */
int oracle_fir_fma(float* y, int32_t y_len, const float* x, int32_t x_len, const float* h,
                   int32_t h_len, int64_t grid, int64_t block) {
    return fir_common(y, y_len, x, x_len, h, h_len, grid, block, 1);
}

static int fir_shard_common(float* y, int64_t y_len, const float* x, int64_t x_len,
                            int64_t halo, const float* h, int32_t taps, int fused) {
    if (taps < 1 || taps > 1024) return E_TAPS;
    if (y_len < 0 || x_len < 0 || halo < 0) return E_LENGTH;
    if (y_len == 0) return 0;
    fir_ctx ctx = {y, y_len, x, x_len, halo, h, taps, fused};
    par_for((y_len + FIR_CHUNK - 1) / FIR_CHUNK, fir_range, &ctx);
    return 0;
}
int oracle_fir_shard(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                     const float* h, int32_t taps) {
    return fir_shard_common(y, y_len, x, x_len, halo, h, taps, 1);
}
int oracle_fir_shard_runcpu(float* y, int64_t y_len, const float* x, int64_t x_len,
                            int64_t halo, const float* h, int32_t taps) {
    return fir_shard_common(y, y_len, x, x_len, halo, h, taps, 0);
}

/* ---- tile graph --------------------------------------------------------- */
/* tile/codegen.go:110-133 renders each operation as one C expression:
 * (k*x), (a+b), (a*b), sqrtf, fabsf, hypotf. Evaluated node by node over the
 * positions [-halo, n). hypotf is gpu.Hypot's definition. */
int oracle_tile_eval(const oracle_tile_node* nodes, int32_t n_nodes, int32_t root, float* out,
                     int32_t n, int32_t halo) {
    if (root < 0 || root >= n_nodes || n < 0 || halo < 0) return E_GRAPH;
    int64_t span = (int64_t)n + halo;
    float** val = (float**)calloc((size_t)n_nodes, sizeof(float*));
    if (!val) return E_GRAPH;
    int rc = 0;
    for (int32_t id = 0; id <= root && rc == 0; id++) {
        const oracle_tile_node* nd = &nodes[id];
        if (nd->kind == 0) continue; /* inputs are read in place */
        float* v = (float*)malloc((size_t)(span > 0 ? span : 1) * sizeof(float));
        if (!v) {
            rc = E_GRAPH;
            break;
        }
        val[id] = v;
#define ARG(j, p) (nodes[(j)].kind == 0 ? nodes[(j)].data[(p)] : val[(j)][(p)])
        for (int64_t p = 0; p < span; p++) {
            switch (nd->kind) {
                case 1: v[p] = nd->scale * ARG(nd->a, p); break;
                case 2: v[p] = ARG(nd->a, p) + ARG(nd->b, p); break;
                case 3: v[p] = ARG(nd->a, p) * ARG(nd->b, p); break;
                case 4: v[p] = go_sqrt32(ARG(nd->a, p)); break;
                case 5: v[p] = fabsf(ARG(nd->a, p)); break;
                case 6: v[p] = oracle_hypot(ARG(nd->a, p), ARG(nd->b, p)); break;
                case 7: {
                    /* Over the whole span, signal values below the span's
                     * start (-halo) reading 0: a window read by another
                     * (chained windows) is read in the halo too. */
                    float acc = 0.0f;
                    for (int32_t k = 0; k < nd->ntaps; k++) {
                        int64_t src = p - k;
                        float t = src >= 0 ? ARG(nd->a, src) : 0.0f;
                        acc = fmaf(nd->taps[k], t, acc);
                    }
                    v[p] = acc;
                    break;
                }
                default: rc = E_GRAPH; break;
            }
            if (rc) break;
        }
#undef ARG
    }
    if (rc == 0) {
        const oracle_tile_node* r = &nodes[root];
        for (int64_t i = 0; i < n; i++)
            out[i] = r->kind == 0 ? r->data[halo + i] : val[root][halo + i];
    }
    for (int32_t id = 0; id < n_nodes; id++) free(val[id]);
    free(val);
    return rc;
}

/* ---- tile reductions -----------------------------------------------------
 * No counterpart in the reference (its PLAN.md, Phase 6, lists tile
 * reductions as future work): the semantics are the library's own, stated
 * in include/simtgo_b200.h (SIMTGO_TILE_SUM ..). Restated here from that
 * statement, element by element, as the check on the GPU tree. */
typedef struct {
    float v;
    int64_t i;
} rval;
#define RED_CHUNK 2048
#define NO_INDEX INT64_MAX

static float f_of(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static uint32_t u_of(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static rval red_id(int kind) {
    rval r = {0.0f, 0};
    if (kind == 1) r.v = f_of(0x7f800000u);
    if (kind >= 2) r.v = f_of(0xff800000u);
    if (kind == 3) r.i = NO_INDEX;
    return r;
}
/* Go's min/max on float32: NaN if either is NaN; -0 < +0. */
static float go_minf(float a, float b) {
    if (a != a || b != b) return f_of(0x7fc00000u);
    if (a < b) return a;
    if (b < a) return b;
    return (u_of(a) >> 31) ? a : b;
}
static float go_maxf(float a, float b) {
    if (a != a || b != b) return f_of(0x7fc00000u);
    if (a > b) return a;
    if (b > a) return b;
    return (u_of(a) >> 31) ? b : a;
}
/* ARGMAX: NaN first, then larger value (+0 above -0), then smaller index. */
static int am_first(rval a, rval b) {
    int na = a.v != a.v, nb = b.v != b.v;
    if (na || nb) return (na && nb) ? a.i < b.i : na;
    if (a.v > b.v) return 1;
    if (b.v > a.v) return 0;
    if ((u_of(a.v) >> 31) != (u_of(b.v) >> 31)) return !(u_of(a.v) >> 31);
    return a.i < b.i;
}
static rval red2(int kind, rval a, rval b) {
    rval r = {0.0f, 0};
    switch (kind) {
        case 0: r.v = a.v + b.v; return r;
        case 1: r.v = go_minf(a.v, b.v); return r;
        case 2: r.v = go_maxf(a.v, b.v); return r;
        default: return am_first(a, b) ? a : b;
    }
}
/* One block of 2048 (value, index) entries, padded with the identity:
 * per lane t ((x[e]+x[e+1])+(x[e+2]+x[e+3]))+((x[f]..)), e = 4t, f = 1024+4t;
 * per warp the butterfly (l with l^16, ^8, ^4, ^2, ^1); then the eight warps
 * as ((w0 w1)(w2 w3))((w4 w5)(w6 w7)). */
static rval red_block(int kind, const rval* x) {
    rval lane[256], w[8];
    for (int t = 0; t < 256; t++) {
        const rval* g0 = x + 4 * t;
        const rval* g1 = x + 1024 + 4 * t;
        lane[t] = red2(kind, red2(kind, red2(kind, g0[0], g0[1]), red2(kind, g0[2], g0[3])),
                       red2(kind, red2(kind, g1[0], g1[1]), red2(kind, g1[2], g1[3])));
    }
    for (int k = 0; k < 8; k++) {
        rval v[32], nv[32];
        memcpy(v, lane + 32 * k, sizeof v);
        for (int m = 16; m >= 1; m >>= 1) {
            for (int l = 0; l < 32; l++) nv[l] = red2(kind, v[l], v[l ^ m]);
            memcpy(v, nv, sizeof v);
        }
        w[k] = v[0];
    }
    return red2(kind, red2(kind, red2(kind, w[0], w[1]), red2(kind, w[2], w[3])),
                red2(kind, red2(kind, w[4], w[5]), red2(kind, w[6], w[7])));
}
/* Level 1: the partial of each block of 2048 values of x (index of x[0] is
 * idx_base) into pv/pi (ceil(n/2048) entries; pi may be null). */
int oracle_tile_reduce_partials(const float* x, int64_t n, int32_t kind, int64_t idx_base,
                                float* pv, int64_t* pi) {
    if (kind < 0 || kind > 3 || n < 0) return E_ARG;
    if (n > 0 && (!x || !pv)) return E_NULL;
    rval* blk = (rval*)malloc(RED_CHUNK * sizeof(rval));
    if (!blk) return E_ARG;
    for (int64_t b = 0; b * RED_CHUNK < n; b++) {
        for (int e = 0; e < RED_CHUNK; e++) {
            const int64_t p = b * RED_CHUNK + e;
            if (p < n) {
                blk[e].v = x[p];
                blk[e].i = idx_base + p;
            } else {
                blk[e] = red_id(kind);
            }
        }
        const rval r = red_block(kind, blk);
        pv[b] = r.v;
        if (pi) pi[b] = r.i;
    }
    free(blk);
    return 0;
}
/* The levels above: m partials (pv, pi) reduced to one value (index -1 for
 * an empty ARGMAX). m = 1 is the result itself; m = 0 the identity. */
int oracle_tile_reduce_levels(const float* pv, const int64_t* pi, int64_t m, int32_t kind,
                              float* value, int64_t* index) {
    if (kind < 0 || kind > 3 || m < 0 || !value) return E_ARG;
    rval* cur = (rval*)malloc((size_t)(m > 0 ? m : 1) * sizeof(rval));
    rval* blk = (rval*)malloc(RED_CHUNK * sizeof(rval));
    if (!cur || !blk) {
        free(cur);
        free(blk);
        return E_ARG;
    }
    for (int64_t e = 0; e < m; e++) {
        cur[e].v = pv[e];
        cur[e].i = pi ? pi[e] : 0;
    }
    rval r = red_id(kind);
    if (m == 0) {
        rval x[RED_CHUNK];
        for (int e = 0; e < RED_CHUNK; e++) x[e] = red_id(kind);
        r = red_block(kind, x);
    }
    while (m > 1) {
        const int64_t nb = (m + RED_CHUNK - 1) / RED_CHUNK;
        for (int64_t b = 0; b < nb; b++) {
            for (int e = 0; e < RED_CHUNK; e++) {
                const int64_t p = b * RED_CHUNK + e;
                blk[e] = p < m ? cur[p] : red_id(kind);
            }
            cur[b] = red_block(kind, blk);
        }
        m = nb;
    }
    if (m == 1) r = cur[0];
    free(cur);
    free(blk);
    if (kind == 0 && r.v != r.v) r.v = f_of(0x7fc00000u); /* NaN payloads differ by platform */
    *value = r.v;
    if (index) *index = (kind == 3 && r.i == NO_INDEX) ? -1 : r.i;
    return 0;
}
int oracle_tile_reduce(const float* x, int64_t n, int32_t kind, int64_t idx_base, float* value,
                       int64_t* index) {
    if (kind < 0 || kind > 3 || n < 0 || !value) return E_ARG;
    const int64_t m = (n + RED_CHUNK - 1) / RED_CHUNK;
    float* pv = (float*)malloc((size_t)(m > 0 ? m : 1) * sizeof(float));
    int64_t* pi = (int64_t*)malloc((size_t)(m > 0 ? m : 1) * sizeof(int64_t));
    int rc = (pv && pi) ? oracle_tile_reduce_partials(x, n, kind, idx_base, pv, pi) : E_ARG;
    if (!rc) rc = oracle_tile_reduce_levels(pv, pi, m, kind, value, index);
    free(pv);
    free(pi);
    return rc;
}
