// elementwise.cu -- the one-sample-per-thread kernels of package kernels:
// VecAdd, Scale, Magnitude (kernels/kernels.go:12-34), MagnitudeFast
// (magnitudefast.go:20), Softclip (softclip.go:25), Classify
// (classify.go:14), BandGain (bandgain.go:42), Quantize (quantize.go:16) and
// Gray (gray.go:34).
//
// B200 design: every kernel is HBM-bound, so one template does the data
// movement for all of them: blocks of 256 threads take contiguous ranges of
// 16-byte vector units, each thread issuing the loads of four units before
// it computes any (64 B of every input stream in flight per thread), with
// L1-bypassing 128-bit loads and evict-first 128-bit stores. Pointers that
// are not 16-byte aligned take a scalar variant of the same arithmetic. The
// arithmetic itself is exact.cuh: the emulator's result, bit for bit. The
// caller's grid*block still bounds which indices are written.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "exact.cuh"

using namespace sgd;

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// ---- the shared data-movement template ------------------------------------
// Op provides: W (elements per vector unit), In (the loaded unit),
// load(v), store(v, in) for unit v, scalar(i) for element i, and
// prologue() (block set-up before the loop; may use shared memory).
//
// Block b takes a contiguous range of about kPerThread units per thread
// (Op::kUnitsPerThread where declared); its threads step through it
// kThreads units apart, kUnroll units per step, so every load and store
// instruction of a warp is one contiguous run. The grid has many more
// blocks than are resident at once, and the hardware hands the next range
// to whichever SM finishes first: on the two-die B200 that measured 5-35%
// faster than a persistent grid striding over the whole array, except for
// Gray's short image (Op::kStrided), which keeps the persistent grid.
// Op::kPipe (where declared true): the loads of a thread's next kUnroll
// units are issued before the stores of the current ones, so they stay in
// flight while it computes.
constexpr int kPerThread = 8;

template <class Op, class = void>
struct Pipelined : std::false_type {};
template <class Op>
struct Pipelined<Op, std::void_t<decltype(Op::kPipe)>> : std::bool_constant<Op::kPipe> {};
template <class Op, class = void>
struct Strided : std::false_type {};
template <class Op>
struct Strided<Op, std::void_t<decltype(Op::kStrided)>> : std::bool_constant<Op::kStrided> {};
template <class Op, class = void>
struct UnitsPerThread : std::integral_constant<int, kPerThread> {};
template <class Op>
struct UnitsPerThread<Op, std::void_t<decltype(Op::kUnitsPerThread)>>
    : std::integral_constant<int, Op::kUnitsPerThread> {};

template <class Op>
__global__ void __launch_bounds__(kThreads) k_vec(Op op, int64_t nvec, int64_t m) {
    op.prologue();
    if constexpr (Strided<Op>::value) {
        const int64_t stride = grid_threads();
        int64_t v = global_tid();
        for (; v + (kUnroll - 1) * stride < nvec; v += kUnroll * stride) {
            typename Op::In in[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) in[u] = op.load(v + u * stride);
#pragma unroll
            for (int u = 0; u < kUnroll; u++) op.store(v + u * stride, in[u]);
        }
        for (; v < nvec; v += stride) op.store(v, op.load(v));
    } else {
        constexpr int64_t kStep = (int64_t)kThreads * kUnroll;
        const int64_t per_block = (nvec + gridDim.x - 1) / gridDim.x;
        const int64_t per = (per_block + kThreads - 1) / kThreads * kThreads;
        const int64_t end = min((int64_t)(blockIdx.x + 1) * per, nvec);
        int64_t v = (int64_t)blockIdx.x * per + threadIdx.x;
        if constexpr (Pipelined<Op>::value) {
            typename Op::In in[kUnroll];
            if (v + (kUnroll - 1) * kThreads < end) {
#pragma unroll
                for (int u = 0; u < kUnroll; u++) in[u] = op.load(v + u * kThreads);
            }
            for (; v + (kUnroll - 1) * kThreads < end; v += kStep) {
                const bool more = v + kStep + (kUnroll - 1) * kThreads < end;
                typename Op::In nx[kUnroll];
                if (more) {
#pragma unroll
                    for (int u = 0; u < kUnroll; u++) nx[u] = op.load(v + kStep + u * kThreads);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; u++) op.store(v + u * kThreads, in[u]);
                if (more) {
#pragma unroll
                    for (int u = 0; u < kUnroll; u++) in[u] = nx[u];
                }
            }
        } else {
            for (; v + (kUnroll - 1) * kThreads < end; v += kStep) {
                typename Op::In in[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; u++) in[u] = op.load(v + u * kThreads);
#pragma unroll
                for (int u = 0; u < kUnroll; u++) op.store(v + u * kThreads, in[u]);
            }
        }
        for (; v < end; v += kThreads) op.store(v, op.load(v));
    }
    for (int64_t i = nvec * Op::W + global_tid(); i < m; i += grid_threads()) op.scalar(i);
}

template <class Op>
__global__ void __launch_bounds__(kThreads) k_scalar(Op op, int64_t m) {
    op.prologue();
    for (int64_t i = global_tid(); i < m; i += grid_threads()) op.scalar(i);
}

// Every argument check has been made by the caller; this is the first step
// that touches the device.
template <class Op>
int run_ew(const char* name, const Op& op, int64_t nvec, int64_t m, bool vec_ok, void* stream) {
    if (m <= 0) return 0;
    const sg::DevInfo* d;
    if (int rc = sg::current_device(&d)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    int64_t blocks;
    if (vec_ok && !Strided<Op>::value) {
        blocks = sg::ceil_div(std::max<int64_t>(nvec, 1),
                              (int64_t)kThreads * UnitsPerThread<Op>::value);
    } else {  // a persistent grid striding over the units (or the elements)
        const int64_t units = vec_ok ? std::max<int64_t>(nvec, 1) : m;
        blocks = std::min<int64_t>(sg::ceil_div(units, (int64_t)kThreads), (int64_t)d->sms * 4);
    }
    sg::before_launch();
    if (vec_ok)
        k_vec<Op><<<(unsigned)blocks, kThreads, 0, s>>>(op, nvec, m);
    else
        k_scalar<Op><<<(unsigned)blocks, kThreads, 0, s>>>(op, m);
    return sg::launch_status(name);
}

struct NoPrologue {
    __device__ void prologue() const {}
};

// ---- VecAdd ----------------------------------------------------------------
struct VecAddOp : NoPrologue {
    float* c;
    const float *a, *b;
    static constexpr int W = 4;
    struct In {
        float4 a, b;
    };
    __device__ In load(int64_t v) const { return {ld_stream_f4(a + 4 * v), ld_stream_f4(b + 4 * v)}; }
    __device__ void store(int64_t v, const In& in) const {
        st_stream_f4(c + 4 * v, make_float4(__fadd_rn(in.a.x, in.b.x), __fadd_rn(in.a.y, in.b.y),
                                            __fadd_rn(in.a.z, in.b.z), __fadd_rn(in.a.w, in.b.w)));
    }
    __device__ void scalar(int64_t i) const { c[i] = __fadd_rn(a[i], b[i]); }
};

// ---- Scale -------------------------------------------------------------------
struct ScaleOp : NoPrologue {
    float* y;
    const float* x;
    float k;
    static constexpr int W = 4;
    using In = float4;
    __device__ In load(int64_t v) const { return ld_stream_f4(x + 4 * v); }
    __device__ void store(int64_t v, const In& a) const {
        st_stream_f4(y + 4 * v, make_float4(__fmul_rn(k, a.x), __fmul_rn(k, a.y),
                                            __fmul_rn(k, a.z), __fmul_rn(k, a.w)));
    }
    __device__ void scalar(int64_t i) const { y[i] = __fmul_rn(k, x[i]); }
};

// ---- Magnitude ----------------------------------------------------------------
struct MagnitudeOp : NoPrologue {
    float* mag;
    const float *re, *im;
    static constexpr int W = 4;
    struct In {
        float4 r, m;
    };
    __device__ In load(int64_t v) const {
        return {ld_stream_f4(re + 4 * v), ld_stream_f4(im + 4 * v)};
    }
    __device__ void store(int64_t v, const In& in) const {
        st_stream_f4(mag + 4 * v, make_float4(hypot_go(in.r.x, in.m.x), hypot_go(in.r.y, in.m.y),
                                              hypot_go(in.r.z, in.m.z), hypot_go(in.r.w, in.m.w)));
    }
    __device__ void scalar(int64_t i) const { mag[i] = hypot_go(re[i], im[i]); }
};

// ---- MagnitudeFast (planar and interleaved) ----------------------------------------
struct MagFastOp : NoPrologue {
    float* mag;
    const float *re, *im;
    float scale;
    static constexpr int W = 4;
    struct In {
        float4 r, m;
    };
    __device__ In load(int64_t v) const {
        return {ld_stream_f4(re + 4 * v), ld_stream_f4(im + 4 * v)};
    }
    __device__ void store(int64_t v, const In& in) const {
        st_stream_f4(mag + 4 * v,
                     make_float4(magfast_go(in.r.x, in.m.x, scale), magfast_go(in.r.y, in.m.y, scale),
                                 magfast_go(in.r.z, in.m.z, scale), magfast_go(in.r.w, in.m.w, scale)));
    }
    __device__ void scalar(int64_t i) const { mag[i] = magfast_go(re[i], im[i], scale); }
};

struct MagFastILOp : NoPrologue {
    float* mag;
    const float* z;
    float scale;
    static constexpr int W = 4;
    struct In {
        float4 a, b;  // (re0, im0, re1, im1), (re2, im2, re3, im3)
    };
    __device__ In load(int64_t v) const {
        return {ld_stream_f4(z + 8 * v), ld_stream_f4(z + 8 * v + 4)};
    }
    __device__ void store(int64_t v, const In& in) const {
        st_stream_f4(mag + 4 * v,
                     make_float4(magfast_go(in.a.x, in.a.y, scale), magfast_go(in.a.z, in.a.w, scale),
                                 magfast_go(in.b.x, in.b.y, scale), magfast_go(in.b.z, in.b.w, scale)));
    }
    __device__ void scalar(int64_t i) const { mag[i] = magfast_go(z[2 * i], z[2 * i + 1], scale); }
};

// ---- Softclip ---------------------------------------------------------------------
struct SoftclipOp : NoPrologue {
    float* y;
    const float* x;
    float t;
    static constexpr int W = 4;
    using In = float4;
    __device__ In load(int64_t v) const { return ld_stream_f4(x + 4 * v); }
    __device__ void store(int64_t v, const In& a) const {
        st_stream_f4(y + 4 * v, make_float4(softclip_go(a.x, t), softclip_go(a.y, t),
                                            softclip_go(a.z, t), softclip_go(a.w, t)));
    }
    __device__ void scalar(int64_t i) const { y[i] = softclip_go(x[i], t); }
};

// ---- Classify ----------------------------------------------------------------------
// The gain depends only on the band the search finds (classify.go:37-48:
// band 0 -> 0.25, 1-2 -> 0.5, 3 -> 0.75, anything else -> 1). A match among
// edges[0..3] decides it; otherwise the band is 4 or later, or -- with no
// match at all -- len(edges), so the no-match gain is the switch applied to
// min(len(edges), 4). Each thread keeps edges[0..3] in registers (a missing
// edge is NaN, which never matches). The bias, the sequential float32 sum of
// every edge (classify.go:50-53), is formed once per block by one thread.
__host__ __device__ inline float classify_gain(int band) {
    switch (band) {
        case 0: return 0.25f;
        case 1:
        case 2: return 0.5f;
        case 3: return 0.75f;
        default: return 1.0f;
    }
}
struct ClassifyOp {
    float* out;
    const float* x;
    const float* edges;
    int32_t n_edges;
    float gain_none;  // classify_gain(len(edges)): the gain when nothing matches
    static constexpr int W = 4;
    using In = float4;
    // Filled by prologue().
    mutable float e0, e1, e2, e3, bias001;

    __device__ void prologue() const {
        __shared__ float s_bias;
        if (threadIdx.x == 0) {
            float b = 0.0f;
            for (int32_t j = 0; j < n_edges; j++) b = __fadd_rn(b, edges[j]);
            s_bias = b;
        }
        const float nan = __int_as_float(0x7fc00000);  // compares false: no match
        e0 = n_edges > 0 ? edges[0] : nan;
        e1 = n_edges > 1 ? edges[1] : nan;
        e2 = n_edges > 2 ? edges[2] : nan;
        e3 = n_edges > 3 ? edges[3] : nan;
        __syncthreads();
        bias001 = __fmul_rn(s_bias, 0.001f);
    }
    __device__ float one(float xv) const {
        const float v = fabsf(xv);
        float gain;
        if (v <= e0)
            gain = 0.25f;
        else if (v <= e1 || v <= e2)
            gain = 0.5f;
        else if (v <= e3)
            gain = 0.75f;
        else
            gain = gain_none;
        return __fadd_rn(__fmul_rn(gain, v), bias001);
    }
    __device__ In load(int64_t v) const { return ld_stream_f4(x + 4 * v); }
    __device__ void store(int64_t v, const In& a) const {
        st_stream_f4(out + 4 * v, make_float4(one(a.x), one(a.y), one(a.z), one(a.w)));
    }
    __device__ void scalar(int64_t i) const { out[i] = one(x[i]); }
};

// ---- BandGain --------------------------------------------------------------------
// kernels/bandgain.go:42-74. The gain is that of the first band, in order,
// whose Upper is >= x[i], else the floor. With U_j = max(Upper_0..Upper_j)
// (NaN uppers skipped; NaN until the first number), that band is the first
// j with x[i] <= U_j: every earlier band has Upper < x[i], so U < x[i]
// there, while U_j >= Upper_j >= x[i]. U is non-decreasing, so a branch-free
// binary search finds j in the same ceil(log2(n+1)) steps on every lane.
// Each block builds U in shared memory (a warp's shuffle prefix max per 32
// bands, carried along), next to gain/4 in float64: float64(sum)/4 *
// float64(gain) + bias is then one fma, as sum*gain/4 of two float32 values
// is exact in float64. A curve longer than kMaxSharedBands is searched in
// order from global memory. Curves of at most K bands (K = 4 or 8) keep U in
// registers, padded with +inf: the band index is then the number of j < K
// with !(x[i] <= U_j), at most n -- K compares and no shared-memory loads.
//
// The 4-tap window x[i-2..i+1] of a vector unit needs x[4v-2], x[4v-1] (the
// previous unit's last two) and x[4v+4] (the next unit's first): the
// neighbouring lanes of the warp hold those units, so they come by shuffle;
// a lane whose neighbour is not there loads them.
constexpr int kMaxSharedBands = 1024;
template <int K>
struct BandGainOp {
    static constexpr int kUnitsPerThread = 32;  // amortises the band-table prologue
    float* y;
    const float* x;
    int64_t x_len;
    const float* bands;  // n_bands (upper, gain) pairs; only 4-byte aligned
    int32_t n_bands;
    float floor_gain;
    float count_f;
    double bias;
    static constexpr int W = 4;
    using In = float4;
    mutable const float* su;   // prefix-max uppers (shared), or null: search in order
    mutable const double* sq;  // gain/4 per band, then the floor's
    mutable int top;           // the largest power of two <= n_bands (0 if none)
    mutable float ur[K > 0 ? K : 1];  // U in registers (K > 0)

    __device__ void prologue() const {
        __shared__ float s_up[kMaxSharedBands];
        __shared__ double s_q[kMaxSharedBands + 1];
        su = nullptr;
        if (n_bands <= kMaxSharedBands) {
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                float carry = __int_as_float(0x7fc00000);  // NaN: no number yet
                for (int j0 = 0; j0 < n_bands; j0 += 32) {
                    const int j = j0 + lane;
                    float u = j < n_bands ? bands[2 * j] : __int_as_float(0x7fc00000);
#pragma unroll
                    for (int d = 1; d < 32; d <<= 1) {
                        const float o = __shfl_up_sync(0xffffffffu, u, d);
                        if (lane >= d) u = fmaxf(u, o);  // fmaxf skips NaN
                    }
                    u = fmaxf(u, carry);
                    if (j < n_bands) s_up[j] = u;
                    carry = __shfl_sync(0xffffffffu, u, 31);
                }
            }
            for (int j = threadIdx.x; j <= n_bands; j += blockDim.x)
                s_q[j] = 0.25 * (double)(j < n_bands ? bands[2 * j + 1] : floor_gain);
            su = s_up;
            sq = s_q;
        }
        top = 0;
        while (2 * top <= n_bands && n_bands > 0) top = top ? 2 * top : 1;
        __syncthreads();
        if (K > 0) {
#pragma unroll
            for (int j = 0; j < (K > 0 ? K : 1); j++)
                ur[j] = j < n_bands ? s_up[j] : __int_as_float(0x7f800000);
        }
    }
    __device__ float xat(int64_t k) const { return (k >= 0 && k < x_len) ? __ldg(x + k) : 0.0f; }
    __device__ float one(float v, float t0, float t1, float t2, float t3) const {
        double q;
        if (K > 0) {
            int pos = 0;
#pragma unroll
            for (int j = 0; j < (K > 0 ? K : 1); j++) pos += !(v <= ur[j]);
            q = sq[min(pos, (int)n_bands)];
        } else if (su) {
            int pos = 0;  // bands before the first with v <= U
            for (int step = top; step > 0; step >>= 1)
                if (pos + step <= n_bands && !(v <= su[pos + step - 1])) pos += step;
            q = sq[pos];
        } else {
            float gain = floor_gain;
            for (int32_t j = 0; j < n_bands; j++)
                if (v <= bands[2 * j]) {
                    gain = bands[2 * j + 1];
                    break;
                }
            q = 0.25 * (double)gain;
        }
        float sum = __fadd_rn(0.0f, t0);
        sum = __fadd_rn(sum, t1);
        sum = __fadd_rn(sum, t2);
        sum = __fadd_rn(sum, t3);
        return __fmul_rn(__double2float_rn(fma((double)sum, q, bias)), count_f);
    }
    __device__ In load(int64_t v) const { return __ldg(reinterpret_cast<const float4*>(x) + v); }
    __device__ void store(int64_t v, const float4& c) const {
        const unsigned mask = __activemask();
        const int lane = threadIdx.x & 31;
        const int vl = (int)v;
        const float pz = __shfl_up_sync(mask, c.z, 1), pw = __shfl_up_sync(mask, c.w, 1);
        const float nx = __shfl_down_sync(mask, c.x, 1);
        const int pv = __shfl_up_sync(mask, vl, 1), nv = __shfl_down_sync(mask, vl, 1);
        const bool have_prev = lane > 0 && ((mask >> (lane - 1)) & 1) && pv == vl - 1;
        const bool have_next = lane < 31 && ((mask >> (lane + 1)) & 1) && nv == vl + 1;
        const float m2 = have_prev ? pz : xat(4 * v - 2);
        const float m1 = have_prev ? pw : xat(4 * v - 1);
        const float p4 = have_next ? nx : xat(4 * v + 4);
        st_stream_f4(y + 4 * v, make_float4(one(c.x, m2, m1, c.x, c.y), one(c.y, m1, c.x, c.y, c.z),
                                            one(c.z, c.x, c.y, c.z, c.w),
                                            one(c.w, c.y, c.z, c.w, p4)));
    }
    __device__ void scalar(int64_t i) const {
        y[i] = one(x[i], xat(i - 2), xat(i - 1), xat(i), xat(i + 1));
    }
};

// ---- Quantize ---------------------------------------------------------------------
struct QuantizeOp : NoPrologue {
    static constexpr bool kPipe = true;
    int32_t* code;
    long long* energy;
    uint8_t* clipped;
    const float* x;
    float step;
    uint32_t seed;
    static constexpr int W = 4;
    using In = float4;
    __device__ void one(int64_t i, float xv, int32_t& q, long long& e, uint32_t& c) const {
        uint32_t h = seed ^ (uint32_t)i;
        h = h * 2654435761u + 1u;
        h ^= h >> 15;
        // float32(int32(h%1024))/1024 - 0.5: the division by a power of two
        // is exact, so it is the same multiply by 2^-10.
        const float jitter = __fsub_rn(__fmul_rn((float)(int32_t)(h % 1024u), 0x1p-10f), 0.5f);
        int32_t qq = go_f32_to_i32(__fadd_rn(__fdiv_rn(xv, step), jitter));
        c = 0;
        if (qq > 127) {
            qq = 127;
            c = 1;
        } else if (qq < -128) {
            qq = -128;
            c = 1;
        }
        q = qq;
        e = (long long)qq * (long long)qq;
    }
    __device__ In load(int64_t v) const { return ld_stream_f4(x + 4 * v); }
    __device__ void store(int64_t v, const In& a) const {
        int4 q;
        longlong2 e01, e23;
        uint32_t c0, c1, c2, c3;
        const int64_t i = 4 * v;
        one(i + 0, a.x, q.x, e01.x, c0);
        one(i + 1, a.y, q.y, e01.y, c1);
        one(i + 2, a.z, q.z, e23.x, c2);
        one(i + 3, a.w, q.w, e23.y, c3);
        // Plain (write-back) stores: 13 of the 17 bytes per element are
        // written, and evict-first stores measured slower on that mix.
        *reinterpret_cast<int4*>(code + i) = q;
        *reinterpret_cast<longlong2*>(energy + i) = e01;
        *reinterpret_cast<longlong2*>(energy + i + 2) = e23;
        *reinterpret_cast<uint32_t*>(clipped + i) = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
    }
    __device__ void scalar(int64_t i) const {
        int32_t q;
        long long e;
        uint32_t c;
        one(i, x[i], q, e, c);
        code[i] = q;
        energy[i] = e;
        clipped[i] = (uint8_t)c;
    }
};

// ---- Gray -----------------------------------------------------------------------
// A vector unit is 16 pixels: 48 bytes of RGB in (three 16-byte loads) and
// 16 bytes of luma out. Two pixels share one 32-bit multiply-add, since
// 77r + 150g + 29b + 128 <= 65408 fits 16 bits (gray.go:12-15, :52).
struct GrayOp : NoPrologue {
    static constexpr bool kStrided = true;
    uint8_t* out;
    const uint8_t* rgb;
    int64_t rgb_len;
    static constexpr int W = 16;
    struct In {
        int4 a, b, c;
    };
    __device__ static uint32_t luma2(uint32_t r, uint32_t g, uint32_t b) {
        // r, g, b hold two channel values in their low bytes of each half.
        const uint32_t y = 77u * r + 150u * g + 29u * b + 0x00800080u;
        return ((y >> 8) & 0xffu) | ((y >> 16) & 0xff00u);
    }
    __device__ In load(int64_t v) const {
        const uint8_t* p = rgb + 48 * v;
        return {ld_stream_i4(p), ld_stream_i4(p + 16), ld_stream_i4(p + 32)};
    }
    __device__ void store(int64_t v, const In& in) const {
        const uint32_t w[12] = {(uint32_t)in.a.x, (uint32_t)in.a.y, (uint32_t)in.a.z,
                                (uint32_t)in.a.w, (uint32_t)in.b.x, (uint32_t)in.b.y,
                                (uint32_t)in.b.z, (uint32_t)in.b.w, (uint32_t)in.c.x,
                                (uint32_t)in.c.y, (uint32_t)in.c.z, (uint32_t)in.c.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            // Four pixels = 12 bytes = words w[3q..3q+2]:
            //   w0 = r0 g0 b0 r1 | w1 = g1 b1 r2 g2 | w2 = b2 r3 g3 b3 (byte 0 first).
            const uint32_t w0 = w[3 * q], w1 = w[3 * q + 1], w2 = w[3 * q + 2];
            // Pixels 0 and 1 in bytes 0 and 2 (the low bytes of the two
            // 16-bit halves), then pixels 2 and 3; bytes 1 and 3 are masked.
            constexpr uint32_t kLo = 0x00ff00ffu;
            const uint32_t r01 = __byte_perm(w0, w1, 0x0300) & kLo;
            const uint32_t g01 = __byte_perm(w0, w1, 0x0401) & kLo;
            const uint32_t b01 = __byte_perm(w0, w1, 0x0502) & kLo;
            const uint32_t r23 = __byte_perm(w1, w2, 0x0502) & kLo;
            const uint32_t g23 = __byte_perm(w1, w2, 0x0603) & kLo;
            const uint32_t b23 = __byte_perm(w1, w2, 0x0704) & kLo;
            const uint32_t y01 = luma2(r01, g01, b01);
            const uint32_t y23 = luma2(r23, g23, b23);
            o[q] = y01 | (y23 << 16);
        }
        st_stream_i4(out + 16 * v, make_int4((int)o[0], (int)o[1], (int)o[2], (int)o[3]));
    }
    __device__ void scalar(int64_t i) const {
        const int64_t j = 3 * i;
        if (j + 2 >= rgb_len) return;
        const int32_t r = rgb[j], g = rgb[j + 1], b = rgb[j + 2];
        out[i] = (uint8_t)((77 * r + 150 * g + 29 * b + 128) >> 8);
    }
};

int nonneg(const char* k, int64_t a, int64_t b = 0, int64_t c = 0, int64_t d = 0) {
    if (a < 0 || b < 0 || c < 0 || d < 0)
        return sg::fail(SIMTGO_EARG, "simt: %s: a slice length is negative", k);
    return 0;
}

}  // namespace

extern "C" {

int simtgo_VecAdd(float* c, int32_t c_len, const float* a, int32_t a_len, const float* b,
                  int32_t b_len, int32_t grid, int32_t block, void* stream) {
    const char* K = "VecAdd";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, c_len, a_len, b_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(c_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "a", a_len, m)) || (rc = sg::check_len(K, "b", b_len, m)) ||
        (rc = sg::check_ptr(K, "c", c, m)) || (rc = sg::check_ptr(K, "a", a, m)) ||
        (rc = sg::check_ptr(K, "b", b, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"c", c, 4LL * c_len, true},
                                  {"a", a, 4LL * a_len, false},
                                  {"b", b, 4LL * b_len, false}})))
        return rc;
    VecAddOp op;
    op.c = c;
    op.a = a;
    op.b = b;
    return run_ew(K, op, m / 4, m, sg::aligned16(c) && sg::aligned16(a) && sg::aligned16(b),
                  stream);
}

int simtgo_Scale(float* y, int32_t y_len, const float* x, int32_t x_len, float k, int32_t grid,
                 int32_t block, void* stream) {
    const char* K = "Scale";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, y_len, x_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(y_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "x", x_len, m)) || (rc = sg::check_ptr(K, "y", y, m)) ||
        (rc = sg::check_ptr(K, "x", x, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"y", y, 4LL * y_len, true}, {"x", x, 4LL * x_len, false}})))
        return rc;
    ScaleOp op;
    op.y = y;
    op.x = x;
    op.k = k;
    return run_ew(K, op, m / 4, m, sg::aligned16(y) && sg::aligned16(x), stream);
}

int simtgo_Magnitude(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                     const float* im, int32_t im_len, int32_t grid, int32_t block, void* stream) {
    const char* K = "Magnitude";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, mag_len, re_len, im_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(mag_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "re", re_len, m)) || (rc = sg::check_len(K, "im", im_len, m)) ||
        (rc = sg::check_ptr(K, "mag", mag, m)) || (rc = sg::check_ptr(K, "re", re, m)) ||
        (rc = sg::check_ptr(K, "im", im, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"mag", mag, 4LL * mag_len, true},
                                  {"re", re, 4LL * re_len, false},
                                  {"im", im, 4LL * im_len, false}})))
        return rc;
    MagnitudeOp op;
    op.mag = mag;
    op.re = re;
    op.im = im;
    return run_ew(K, op, m / 4, m, sg::aligned16(mag) && sg::aligned16(re) && sg::aligned16(im),
                  stream);
}

int simtgo_MagnitudeFast(float* mag, int32_t mag_len, const float* re, int32_t re_len,
                         const float* im, int32_t im_len, float scale, int32_t grid,
                         int32_t block, void* stream) {
    const char* K = "MagnitudeFast";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, mag_len, re_len, im_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(mag_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "re", re_len, m)) || (rc = sg::check_len(K, "im", im_len, m)) ||
        (rc = sg::check_ptr(K, "mag", mag, m)) || (rc = sg::check_ptr(K, "re", re, m)) ||
        (rc = sg::check_ptr(K, "im", im, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"mag", mag, 4LL * mag_len, true},
                                  {"re", re, 4LL * re_len, false},
                                  {"im", im, 4LL * im_len, false}})))
        return rc;
    MagFastOp op;
    op.mag = mag;
    op.re = re;
    op.im = im;
    op.scale = scale;
    return run_ew(K, op, m / 4, m, sg::aligned16(mag) && sg::aligned16(re) && sg::aligned16(im),
                  stream);
}

int simtgo_MagnitudeFast_interleaved(float* mag, int32_t mag_len, const float* z, int32_t z_len,
                                     float scale, int32_t grid, int32_t block, void* stream) {
    const char* K = "MagnitudeFast_interleaved";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, mag_len, z_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(mag_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "z", z_len, 2 * m)) || (rc = sg::check_ptr(K, "mag", mag, m)) ||
        (rc = sg::check_ptr(K, "z", z, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"mag", mag, 4LL * mag_len, true}, {"z", z, 4LL * z_len, false}})))
        return rc;
    MagFastILOp op;
    op.mag = mag;
    op.z = z;
    op.scale = scale;
    return run_ew(K, op, m / 4, m, sg::aligned16(mag) && sg::aligned16(z), stream);
}

int simtgo_Softclip(float* y, int32_t y_len, const float* x, int32_t x_len, float threshold,
                    int32_t grid, int32_t block, void* stream) {
    const char* K = "Softclip";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, y_len, x_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(y_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "x", x_len, m)) || (rc = sg::check_ptr(K, "y", y, m)) ||
        (rc = sg::check_ptr(K, "x", x, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"y", y, 4LL * y_len, true}, {"x", x, 4LL * x_len, false}})))
        return rc;
    SoftclipOp op;
    op.y = y;
    op.x = x;
    op.t = threshold;
    return run_ew(K, op, m / 4, m, sg::aligned16(y) && sg::aligned16(x), stream);
}

int simtgo_Classify(float* out, int32_t out_len, const float* x, int32_t x_len,
                    const float* edges, int32_t edges_len, int32_t grid, int32_t block,
                    void* stream) {
    const char* K = "Classify";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, out_len, x_len, edges_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(out_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "x", x_len, m)) || (rc = sg::check_ptr(K, "out", out, m)) ||
        (rc = sg::check_ptr(K, "x", x, m)) || (rc = sg::check_ptr(K, "edges", edges, edges_len)))
        return rc;
    if ((rc = sg::check_alias(K, {{"out", out, 4LL * out_len, true},
                                  {"x", x, 4LL * x_len, false},
                                  {"edges", edges, 4LL * edges_len, false}})))
        return rc;
    ClassifyOp op;
    op.out = out;
    op.x = x;
    op.edges = edges;
    op.n_edges = edges_len;
    op.gain_none = classify_gain(edges_len);
    return run_ew(K, op, m / 4, m, sg::aligned16(out) && sg::aligned16(x), stream);
}

int simtgo_BandGain(float* y, int32_t y_len, const float* x, int32_t x_len,
                    const simtgo_band* bands, int32_t bands_len, const simtgo_shape* cfg,
                    int32_t grid, int32_t block, void* stream) {
    const char* K = "BandGain";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, y_len, x_len, bands_len))) return rc;
    if (!cfg) return sg::fail(SIMTGO_ENULL, "simt: BandGain: cfg (the Shape) is null");
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(y_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "x", x_len, m)) || (rc = sg::check_ptr(K, "y", y, m)) ||
        (rc = sg::check_ptr(K, "x", x, m)) || (rc = sg::check_ptr(K, "bands", bands, bands_len)))
        return rc;
    if ((rc = sg::check_alias(K, {{"y", y, 4LL * y_len, true},
                                  {"x", x, 4LL * x_len, false},
                                  {"bands", bands, 8LL * bands_len, false}})))
        return rc;
    auto run = [&](auto op) {
        op.y = y;
        op.x = x;
        op.x_len = x_len;
        op.bands = reinterpret_cast<const float*>(bands);
        op.n_bands = bands_len;
        op.floor_gain = cfg->floor_gain;
        op.count_f = (float)cfg->count;  // float32(cfg.Count): int32 -> nearest float32
        op.bias = cfg->bias;
        return run_ew(K, op, m / 4, m, sg::aligned16(y) && sg::aligned16(x), stream);
    };
    if (bands_len <= 4) return run(BandGainOp<4>());
    if (bands_len <= 8) return run(BandGainOp<8>());
    return run(BandGainOp<0>());
}

int simtgo_Quantize(int32_t* code, int32_t code_len, int64_t* energy, int32_t energy_len,
                    uint8_t* clipped, int32_t clipped_len, const float* x, int32_t x_len,
                    float step, uint32_t seed, int32_t grid, int32_t block, void* stream) {
    const char* K = "Quantize";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, code_len, energy_len, clipped_len, x_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(code_len, nt);
    if (m <= 0) return 0;
    if ((rc = sg::check_len(K, "energy", energy_len, m)) ||
        (rc = sg::check_len(K, "clipped", clipped_len, m)) ||
        (rc = sg::check_len(K, "x", x_len, m)) || (rc = sg::check_ptr(K, "code", code, m)) ||
        (rc = sg::check_ptr(K, "energy", energy, m)) ||
        (rc = sg::check_ptr(K, "clipped", clipped, m)) || (rc = sg::check_ptr(K, "x", x, m)))
        return rc;
    if ((rc = sg::check_alias(K, {{"code", code, 4LL * code_len, true},
                                  {"energy", energy, 8LL * energy_len, true},
                                  {"clipped", clipped, (int64_t)clipped_len, true},
                                  {"x", x, 4LL * x_len, false}})))
        return rc;
    QuantizeOp op;
    op.code = code;
    op.energy = reinterpret_cast<long long*>(energy);
    op.clipped = clipped;
    op.x = x;
    op.step = step;
    op.seed = seed;
    const bool vec = sg::aligned16(code) && sg::aligned16(energy) && sg::aligned16(x) &&
                     (((uintptr_t)clipped & 3u) == 0);
    return run_ew(K, op, m / 4, m, vec, stream);
}

int simtgo_Gray(uint8_t* out, int32_t out_len, const uint8_t* rgb, int32_t rgb_len, int32_t grid,
                int32_t block, void* stream) {
    const char* K = "Gray";
    sg::clear_error();
    int64_t nt;
    int rc;
    if ((rc = nonneg(K, out_len, rgb_len))) return rc;
    if ((rc = sg::launch_extent_1d(K, grid, block, 0, &nt))) return rc;
    const int64_t m = std::min<int64_t>(out_len, nt);
    if (m <= 0) return 0;
    // Pixels whose three channels lie inside rgb are written; the rest are
    // skipped (gray.go:44-47), so nothing is out of range.
    const int64_t px = std::min<int64_t>(m, rgb_len / 3);
    if ((rc = sg::check_ptr(K, "out", out, m)) || (rc = sg::check_ptr(K, "rgb", rgb, px)))
        return rc;
    if ((rc = sg::check_alias(K, {{"out", out, (int64_t)out_len, true},
                                  {"rgb", rgb, (int64_t)rgb_len, false}})))
        return rc;
    GrayOp op;
    op.out = out;
    op.rgb = rgb;
    op.rgb_len = rgb_len;
    const int64_t nvec = std::min<int64_t>(m / 16, (int64_t)rgb_len / 48);
    return run_ew(K, op, nvec, m, sg::aligned16(out) && sg::aligned16(rgb), stream);
}

}  // extern "C"
