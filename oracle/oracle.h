/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY. A CPU restatement of what simtgo's
 * gpu.RunCPU emulator (gpu/gpu.go:244-431) computes for each hot-path kernel
 * of package kernels and for the tile track's fused graph.
 *
 * Only the test suite, the smoke check and the benchmark's CPU-baseline leg
 * use this library, and only as the reference result or as the timed CPU
 * baseline. The product (libsimtgo_b200.so) neither links nor calls it.
 *
 * Every function mirrors the matching simtgo_* entry point of
 * include/simtgo_b200.h minus the stream, computes on the host, and returns
 * the same status codes (0, or a negative SIMTGO_E* value where gpu.RunCPU
 * would have panicked with an index out of range).
 *
 * Built with -ffp-contract=off: the amd64 Go compiler never fuses a*b+c, so
 * every float operation here is rounded on its own, as in the emulator.
 *
 * Parity is pinned two ways: against golden vectors made by the reference's
 * own generated kernels (the kernels/prebuilt .cu files) compiled for the host
 * (oracle/_ref, tests/golden/make_golden.py), and against the known-answer
 * tests restated from the reference's parity tests.
 */
#ifndef SIMTGO_ORACLE_H
#define SIMTGO_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Worker threads for the block loop (runCPU's pool, gpu/gpu.go:319-356). */
void oracle_set_threads(int n);
int oracle_get_threads(void);

/* gpu.Hypot (gpu/math.go:17) = float32(math.Hypot(float64(x), float64(y))). */
float oracle_hypot(float x, float y);

int oracle_vecadd(float* c, int32_t c_len, const float* a, int32_t a_len,
                  const float* b, int32_t b_len, int64_t grid, int64_t block);
int oracle_scale(float* y, int32_t y_len, const float* x, int32_t x_len, float k,
                 int64_t grid, int64_t block);
int oracle_magnitude(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                     const float* im, int32_t im_len, int64_t grid, int64_t block);
int oracle_magnitudefast(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                         const float* im, int32_t im_len, float scale,
                         int64_t grid, int64_t block);
int oracle_magnitudefast_interleaved(float* mag, int32_t mag_len, const float* z,
                                     int32_t z_len, float scale, int64_t grid, int64_t block);
int oracle_softclip(float* y, int32_t y_len, const float* x, int32_t x_len, float threshold,
                    int64_t grid, int64_t block);
int oracle_classify(float* out, int32_t out_len, const float* x, int32_t x_len,
                    const float* edges, int32_t edges_len, int64_t grid, int64_t block);

typedef struct oracle_band { float upper; float gain; } oracle_band;
typedef struct oracle_shape { float floor_gain; int32_t count; double bias; } oracle_shape;
int oracle_bandgain(float* y, int32_t y_len, const float* x, int32_t x_len,
                    const oracle_band* bands, int32_t bands_len, const oracle_shape* cfg,
                    int64_t grid, int64_t block);
int oracle_quantize(int32_t* code, int32_t code_len, int64_t* energy, int32_t energy_len,
                    uint8_t* clipped, int32_t clipped_len, const float* x, int32_t x_len,
                    float step, uint32_t seed, int64_t grid, int64_t block);
int oracle_gray(uint8_t* out, int32_t out_len, const uint8_t* rgb, int32_t rgb_len,
                int64_t grid, int64_t block);
int oracle_histogram(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                     int64_t grid, int64_t block);
int oracle_transpose(float* out, int32_t out_len, const float* in, int32_t in_len,
                     int32_t w, int32_t h, int64_t grid_x, int64_t grid_y,
                     int64_t block_x, int64_t block_y);
int oracle_warpreducesum(float* out, int32_t out_len, const float* x, int32_t x_len,
                         int64_t grid, int64_t block);
/* FIR as gpu.RunCPU computes it: acc = acc + h[k]*x, each rounded. */
int oracle_fir(float* y, int32_t y_len, const float* x, int32_t x_len,
               const float* h, int32_t h_len, int64_t grid, int64_t block);
/* FIR in the device's order: acc = fma(h[k], x, acc), k = 0..taps-1. */
int oracle_fir_fma(float* y, int32_t y_len, const float* x, int32_t x_len,
                   const float* h, int32_t h_len, int64_t grid, int64_t block);
/* One shard of a long FIR in the device's fma order (simtgo_FIR_shard). */
int oracle_fir_shard(float* y, int64_t y_len, const float* x, int64_t x_len, int64_t halo,
                     const float* h, int32_t taps);
/* The same shard with the emulator's separately rounded multiply and add. */
int oracle_fir_shard_runcpu(float* y, int64_t y_len, const float* x, int64_t x_len,
                            int64_t halo, const float* h, int32_t taps);
/* Histogram with a launch-sized tile of tile_len bins (LaunchShared on the
 * DynProbe body): adds the counts of x[i] in [0, tile_len) into bins[k] for
 * k < min(tile_len, bins_len). */
int oracle_histogram_dyn(int32_t* bins, int32_t bins_len, const int32_t* x, int32_t x_len,
                         int32_t tile_len, int64_t grid, int64_t block);
/* Histogram over a 64-bit extent (simtgo_Histogram_shard). */
int oracle_histogram_shard(int32_t* bins, int32_t bins_len, const int32_t* x, int64_t x_len);

/* ---- tile graph --------------------------------------------------------
 * A recorded graph as a node table in creation order (tile/tile.go:40-49).
 * kind: 0 input, 1 scale, 2 add, 3 mul, 4 sqrt, 5 abs, 6 hypot, 7 fir.
 * An input's data is `data` (n floats, with `halo` preceding elements for a
 * shard evaluation). A FIR node's taps are `taps` (ntaps floats). Nodes are
 * evaluated one at a time, which is what the fused kernel computes too:
 * every operation is rounded on its own; a FIR tile value at an index before
 * the start of the signal (or of the shard's halo) is 0 (tile/codegen.go:
 * 80-108), and its accumulation is fma(h[k], tile, acc) in k order, as the
 * reference's NVRTC build contracts `v += h[k]*tile[...]`. A FIR node's
 * values exist over the whole span, halo included, so a FIR may read
 * another (the library's opt-in chained windows). */
typedef struct oracle_tile_node {
    int32_t kind;
    int32_t a, b;
    float scale;
    const float* data;
    const float* taps;
    int32_t ntaps;
} oracle_tile_node;
int oracle_tile_eval(const oracle_tile_node* nodes, int32_t n_nodes, int32_t root,
                     float* out, int32_t n, int32_t halo);

/* ---- tile reductions ----------------------------------------------------
 * No counterpart in the reference: the library's own SUM (0), MIN (1),
 * MAX (2) and ARGMAX (3) over n values x (index of x[0] = idx_base), in the
 * tree include/simtgo_b200.h states. _partials gives the first level (one
 * entry per block of 2048 values), _levels the rest. */
int oracle_tile_reduce(const float* x, int64_t n, int32_t kind, int64_t idx_base, float* value,
                       int64_t* index);
int oracle_tile_reduce_partials(const float* x, int64_t n, int32_t kind, int64_t idx_base,
                                float* pv, int64_t* pi);
int oracle_tile_reduce_levels(const float* pv, const int64_t* pi, int64_t m, int32_t kind,
                              float* value, int64_t* index);

#ifdef __cplusplus
}
#endif
#endif
