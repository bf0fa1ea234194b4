// exact.cuh -- device arithmetic that reproduces gpu.RunCPU bit for bit.
//
// The emulator runs the Go kernel bodies on amd64, where every float32 and
// float64 operation is rounded on its own (no contraction) and gpu.Sqrt /
// gpu.Hypot are the float64 functions rounded once to float32
// (gpu/math.go:11-17). Everything here therefore uses the _rn intrinsics
// explicitly; the library is also compiled with --fmad=false.
#pragma once
#ifndef __CUDACC_RTC__
#include <cuda_runtime.h>
#include <stdint.h>
#endif

namespace sgd {

// Go's float32 -> int32 conversion on amd64 (CVTTSS2SL): truncation toward
// zero, and INT32_MIN for NaN or a value outside [-2^31, 2^31).
__device__ __forceinline__ int32_t go_f32_to_i32(float f) {
    return (f >= -2147483648.0f && f < 2147483648.0f) ? __float2int_rz(f) : INT32_MIN;
}

// math.Hypot's steps (Go's pure-Go and amd64 versions agree): p = max(|x|,|y|),
// q = min; +Inf if either is infinite, NaN if either is NaN, 0 if p == 0,
// else p * Sqrt(1 + (q/p)^2), each step a correctly rounded float64
// operation. Used for the rare inputs the fast path below cannot decide.
static __device__ __noinline__ float hypot_go_exact(float xf, float yf) {
    double p = fabs((double)xf), q = fabs((double)yf);
    if (isinf(p) || isinf(q)) return __int_as_float(0x7f800000);
    if (isnan(p) || isnan(q)) return __int_as_float(0x7fc00000);
    if (p < q) {
        double t = p;
        p = q;
        q = t;
    }
    if (p == 0.0) return 0.0f;
    q = __ddiv_rn(q, p);
    double s = __dadd_rn(1.0, __dmul_rn(q, q));
    return __double2float_rn(__dmul_rn(p, __dsqrt_rn(s)));
}

// gpu.Hypot(x, y) = float32(math.Hypot(float64(x), float64(y))), bit-exact.
//
// Fast path (own method): s = x^2 + y^2 in float64 (x^2 and y^2 are exact
// there; the sum is rounded once), an approximate reciprocal square root of
// s from the SFU, and one Newton-Raphson correction in float64
// (g1 = g0 + r0/2 * (s - g0^2), g0 = s*r0). rsqrtf is within 2 ulp
// (relative 2^-22), so the corrected value is within 1.5 * 2^-44 (relative)
// of sqrt(s), i.e. under 800 float64 ulps of hypot. math.Hypot's float64
// result lies within a few float64 ulps of hypot as well, so both round to
// the same float32 unless hypot sits near a float32 rounding midpoint. That
// case -- the 29 bits that rounding discards are within 4096 of the midpoint
// pattern -- and any input outside [2^-60, 2^60] (where s would leave
// float32's exponent range), zero, infinity or NaN take hypot_go_exact. The
// fraction of random inputs that do is about 2^-16.
__device__ __forceinline__ float hypot_go(float x, float y) {
    const float ax = fabsf(x), ay = fabsf(y);
    const float p = fmaxf(ax, ay);
    // NaN fails both comparisons, so it takes the exact path too.
    if (!(p >= 0x1p-60f && p <= 0x1p60f)) return hypot_go_exact(x, y);
    const double dx = (double)x, dy = (double)y;
    const double s = fma(dx, dx, __dmul_rn(dy, dy));
    const float r0f = rsqrtf(__double2float_rn(s));
    const double r0 = (double)r0f;
    const double g0 = __dmul_rn(s, r0);
    const double e = fma(-g0, g0, s);
    const double g1 = fma(0.5 * r0, e, g0);
    const unsigned long long bits = (unsigned long long)__double_as_longlong(g1);
    const int32_t low = (int32_t)(bits & 0x1fffffffull) - 0x10000000;
    if (low >= -4096 && low <= 4096) return hypot_go_exact(x, y);
    return __double2float_rn(g1);
}

// Four gpu.Hypot values at once, bit for bit as hypot_go: the fast path of
// all four first, with no branch between them, so that their float64 chains
// interleave (one value's chain is about nine dependent float64 steps), then
// hypot_go_exact for the rare values the fast path cannot decide.
__device__ __forceinline__ float4 hypot_go4(float4 x, float4 y) {
    const float xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
    float r[4];
    bool slow[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float p = fmaxf(fabsf(xs[i]), fabsf(ys[i]));
        const double dx = (double)xs[i], dy = (double)ys[i];
        const double s = fma(dx, dx, __dmul_rn(dy, dy));
        const double r0 = (double)rsqrtf(__double2float_rn(s));
        const double g0 = __dmul_rn(s, r0);
        const double g1 = fma(0.5 * r0, fma(-g0, g0, s), g0);
        const int32_t low =
            (int32_t)((unsigned long long)__double_as_longlong(g1) & 0x1fffffffull) - 0x10000000;
        // NaN fails both range comparisons.
        slow[i] = !(p >= 0x1p-60f && p <= 0x1p60f) || (low >= -4096 && low <= 4096);
        r[i] = __double2float_rn(g1);
    }
    if (slow[0] || slow[1] || slow[2] || slow[3]) {
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (slow[i]) r[i] = hypot_go_exact(xs[i], ys[i]);
    }
    return make_float4(r[0], r[1], r[2], r[3]);
}

// kernels/softclip.go:11-23.
__device__ __forceinline__ float softclip_go(float v, float t) {
    const float a = fabsf(v);
    if (a <= t) return v;
    const float over = __fsub_rn(a, t);
    const float shaped = __fadd_rn(t, __fdiv_rn(over, __fadd_rn(1.0f, over)));
    return v < 0.0f ? -shaped : shaped;
}

// kernels/magnitudefast.go:24-25: Sqrt(r*r + m*m) / scale, each step rounded.
__device__ __forceinline__ float magfast_go(float r, float m, float scale) {
    const float s = __fadd_rn(__fmul_rn(r, r), __fmul_rn(m, m));
    return __fdiv_rn(__fsqrt_rn(s), scale);
}

}  // namespace sgd
