// transpose.cu -- Transpose (kernels/transpose.go:15-38).
//
// The reference stages a 16x16 tile per 256-thread block and reads it back
// down its columns, tile[tx*16+ty], which on a 32-bank shared memory is an
// 8-way bank conflict, and writes 64-byte row segments. Here a block of 256
// threads moves a 64x64 tile: 16-byte loads of input rows (each warp reads
// four 128-byte row segments), a shared tile padded to 65 floats per row so
// that both the row writes and the column reads are conflict-free, and
// 16-byte stores of output rows (each warp writes four 128-byte segments).
// Edge tiles and matrices whose rows are not 16-byte multiples use the same
// tile with scalar accesses.
//
// Semantics kept: only the rectangle the caller's grid covered is moved,
// out[x*h + y] = in[y*w + x] for x < min(w, 16*grid_x), y < min(h, 16*grid_y).
#include <algorithm>

#include "common.cuh"

using namespace sgd;

namespace {

constexpr int kT = 64;       // tile edge
constexpr int kPitch = 65;   // padded shared row
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) k_transpose(float* __restrict__ out,
                                                        const float* __restrict__ in, int64_t w,
                                                        int64_t h, int64_t xcov, int64_t ycov,
                                                        int64_t tiles_x, bool vec_in,
                                                        bool vec_out) {
    __shared__ float tile[kT * kPitch];
    const int tid = threadIdx.x;
    const int64_t tx = blockIdx.x % tiles_x, ty = blockIdx.x / tiles_x;
    const int64_t x0 = tx * kT, y0 = ty * kT;  // input column / row origin
    const bool full = (x0 + kT <= xcov) && (y0 + kT <= ycov);

    // Load: lane -> (q = lane % 8: float4 within a 128-byte half-row,
    // r = lane / 8 + 4*warp: row); eight passes cover 64 rows x 16 float4s.
    {
        const int q = tid & 7, rr = tid >> 3;  // rr in [0, 32)
        if (full && vec_in) {
            float4 v[4];
#pragma unroll
            for (int p = 0; p < 4; p++) {
                // p selects (row half, column half): rows rr and rr+32,
                // float4 q and q+8.
                const int r = rr + 32 * (p >> 1), c4 = q + 8 * (p & 1);
                v[p] = ld_stream_f4(in + (y0 + r) * w + x0 + 4 * c4);
            }
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const int r = rr + 32 * (p >> 1), c4 = q + 8 * (p & 1);
                float* t = tile + r * kPitch + 4 * c4;
                t[0] = v[p].x;
                t[1] = v[p].y;
                t[2] = v[p].z;
                t[3] = v[p].w;
            }
        } else {
            for (int k = tid; k < kT * kT; k += kThreads) {
                const int r = k / kT, c = k % kT;
                const int64_t y = y0 + r, x = x0 + c;
                if (y < ycov && x < xcov) tile[r * kPitch + c] = in[y * w + x];
            }
        }
    }
    __syncthreads();
    // Store: output row oc = input column; lane -> (q = lane % 8: float4 of
    // output row, oc = lane / 8 + 4*warp + 32*pass); bank of a column read
    // = (4q + i + oc) mod 32, distinct over the warp.
    {
        const int q = tid & 7, oo = tid >> 3;  // oo in [0, 32)
        if (full && vec_out) {
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const int oc = oo + 32 * (p >> 1), r4 = q + 8 * (p & 1);
                const float* t = tile + (4 * r4) * kPitch + oc;
                const float4 v = make_float4(t[0], t[kPitch], t[2 * kPitch], t[3 * kPitch]);
                st_stream_f4(out + (x0 + oc) * h + y0 + 4 * r4, v);
            }
        } else {
            for (int k = tid; k < kT * kT; k += kThreads) {
                const int oc = k / kT, r = k % kT;
                const int64_t x = x0 + oc, y = y0 + r;
                if (y < ycov && x < xcov) out[x * h + y] = tile[r * kPitch + oc];
            }
        }
    }
}

}  // namespace

extern "C" int simtgo_Transpose(float* out, int32_t out_len, const float* in, int32_t in_len,
                                int32_t w, int32_t h, int32_t grid_x, int32_t grid_y,
                                int32_t block_x, int32_t block_y, void* stream) {
    const char* K = "Transpose";
    sg::clear_error();
    const sg::DevInfo* d;
    int rc;
    if (out_len < 0 || in_len < 0) return sg::fail(SIMTGO_EARG, "simt: %s: negative length", K);
    if (block_x <= 0 || block_y <= 0 || (int64_t)block_x * block_y > 1024 || grid_x <= 0 ||
        grid_y <= 0 || grid_y > 65535)
        return sg::fail(SIMTGO_ELAUNCH, "simt: %s: grid (%d,%d) block (%d,%d) is not launchable",
                        K, grid_x, grid_y, block_x, block_y);
    if ((int64_t)block_x * block_y != 256)
        return sg::fail(SIMTGO_EBLOCK, "simt: %s requires block == %d, got %d", K, 256,
                        block_x * block_y);
    if (block_x != 16 || block_y != 16)
        return sg::fail(SIMTGO_EBLOCK,
                        "simt: %s: its tile is 16x16; a %dx%d block indexes past it "
                        "(gpu.RunCPU panics: index out of range)",
                        K, block_x, block_y);
    const int64_t xcov = std::min<int64_t>(w, 16LL * grid_x);
    const int64_t ycov = std::min<int64_t>(h, 16LL * grid_y);
    if (xcov <= 0 || ycov <= 0) return 0;
    const int64_t need_in = (ycov - 1) * (int64_t)w + xcov;
    const int64_t need_out = (xcov - 1) * (int64_t)h + ycov;
    if ((rc = sg::check_len(K, "in", in_len, need_in)) ||
        (rc = sg::check_len(K, "out", out_len, need_out)) ||
        (rc = sg::check_ptr(K, "out", out, need_out)) || (rc = sg::check_ptr(K, "in", in, need_in)))
        return rc;
    if ((rc = sg::check_alias(K, {{"out", out, 4LL * out_len, true},
                                  {"in", in, 4LL * in_len, false}})))
        return rc;
    const int64_t tiles_x = sg::ceil_div(xcov, kT), tiles_y = sg::ceil_div(ycov, kT);
    const int64_t tiles = tiles_x * tiles_y;
    if (tiles > 0x7fffffffLL) return sg::fail(SIMTGO_ESIZE, "simt: %s: matrix too large", K);
    if ((rc = sg::current_device(&d))) return rc;
    const bool vec_in = sg::aligned16(in) && (w % 4 == 0);
    const bool vec_out = sg::aligned16(out) && (h % 4 == 0);
    sg::before_launch();
    k_transpose<<<(unsigned)tiles, kThreads, 0, (cudaStream_t)stream>>>(out, in, w, h, xcov, ycov,
                                                                       tiles_x, vec_in, vec_out);
    return sg::launch_status(K);
}
